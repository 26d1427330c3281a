// Host helpers shared by the launch translation units (declared in launch.cuh).
#include <cudaTypedefs.h>

#include <cstdlib>
#include <cstring>

#include "launch.cuh"

namespace va {

// Device error word of the library (first writer wins; read and cleared by
// va_device_error). Every translation unit's kernels write this one word.
__device__ int g_device_error = 0;

namespace host {

namespace {
thread_local int t_last_cuda_error = 0;
}

int cuda_fail(cudaError_t e) {
    t_last_cuda_error = (int)e;
    return VA_ERR_CUDA;
}

int last_cuda_error() { return t_last_cuda_error; }

int current_device(int* dev) {
    VA_CUDA(cudaGetDevice(dev));
    if (*dev < 0 || *dev >= kMaxDevices) return VA_ERR_UNSUPPORTED;
    return VA_OK;
}

int sm_count(int dev) {
    static int cache[kMaxDevices] = {0};
    if (cache[dev] == 0) {
        int n = 0;
        if (cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess || n <= 0) n = 148;
        cache[dev] = n;
    }
    return cache[dev];
}

// Measured on B200: at D = 128 the tensor-core tile kernels for batch-1
// decode of q3+/q4+/q8+ (decode_tc.cuh) and grouped-query decode of q4+ with
// 2, 4 or 8 query heads per KV head (decode_tcg.cuh); for other grouped-query
// shapes the tensor-core consumer of decode_mma.cuh; otherwise the integer
// dot-product consumer.
Consumer pick_consumer(Kind k, int D, int G) {
    static const int v = [] {
        const char* e = std::getenv("VOLTATTN_CONSUMER");
        if (e && std::strcmp(e, "dp") == 0) return 0;
        if (e && std::strcmp(e, "mma") == 0) return 1;
        if (e && std::strcmp(e, "tc") == 0) return 2;
        return -1;
    }();
    const bool tc_ok =
        D == 128 && ((G == 1 && (k == Kind::Q3 || k == Kind::Q4 || k == Kind::Q8)) ||
                     ((G == 2 || G == 4 || G == 8) && k == Kind::Q4));
    if (v == 0) return Consumer::kDp;
    if (v == 1) return Consumer::kMma;
    if (v == 2 && tc_ok) return Consumer::kTc;
    if (tc_ok) return Consumer::kTc;
    return G >= 2 ? Consumer::kMma : Consumer::kDp;
}

namespace {
PFN_cuTensorMapEncodeTiled_v12000 tensor_map_encoder() {
    static PFN_cuTensorMapEncodeTiled_v12000 fn = [] {
        void* f = nullptr;
        cudaDriverEntryPointQueryResult q;
        if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &f, cudaEnableDefault, &q) != cudaSuccess ||
            q != cudaDriverEntryPointSuccess)
            f = nullptr;
        return reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(f);
    }();
    return fn;
}
}  // namespace

// Swizzle span = row bytes (64 or 128; other widths, the 48-byte q3 rows,
// unswizzled), zero fill past the last row.
int encode_rows_map(CUtensorMap* m, const void* base, long long rows, int row_bytes, int box_rows) {
    const auto enc = tensor_map_encoder();
    if (!enc) return VA_ERR_UNSUPPORTED;
    const cuuint64_t dims[2] = {(cuuint64_t)row_bytes, (cuuint64_t)rows};
    const cuuint64_t strides[1] = {(cuuint64_t)row_bytes};
    const cuuint32_t box[2] = {(cuuint32_t)row_bytes, (cuuint32_t)box_rows};
    const cuuint32_t estr[2] = {1, 1};
    const CUtensorMapSwizzle sw = row_bytes == 128  ? CU_TENSOR_MAP_SWIZZLE_128B
                                  : row_bytes == 64 ? CU_TENSOR_MAP_SWIZZLE_64B
                                                    : CU_TENSOR_MAP_SWIZZLE_NONE;
    const CUresult r = enc(m, CU_TENSOR_MAP_DATA_TYPE_UINT8, 2, const_cast<void*>(base), dims, strides, box, estr,
                           CU_TENSOR_MAP_INTERLEAVE_NONE, sw, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                           CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    return r == CUDA_SUCCESS ? VA_OK : VA_ERR_UNSUPPORTED;
}

// fp16 rows of 128 elements ([rows][128], 256-byte stride), boxes of 64
// elements (128 bytes, the 128-byte swizzle span) by box_rows rows.
int encode_f16_rows_map(CUtensorMap* m, const void* base, long long rows, int box_rows) {
    const auto enc = tensor_map_encoder();
    if (!enc) return VA_ERR_UNSUPPORTED;
    const cuuint64_t dims[2] = {128, (cuuint64_t)rows};
    const cuuint64_t strides[1] = {256};
    const cuuint32_t box[2] = {64, (cuuint32_t)box_rows};
    const cuuint32_t estr[2] = {1, 1};
    const CUresult r = enc(m, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 2, const_cast<void*>(base), dims, strides, box, estr,
                           CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
                           CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    return r == CUDA_SUCCESS ? VA_OK : VA_ERR_UNSUPPORTED;
}

}  // namespace host
}  // namespace va
