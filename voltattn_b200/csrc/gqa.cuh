// Batched grouped-query decode (placeholder until the kernel lands).
#pragma once

#include "../../include/voltattn.h"
#include "common.cuh"

namespace va {

inline size_t gqa_workspace_bytes(int B, int Hq, int D, int S) {
    if (B < 1 || Hq < 1 || D < 1 || S < 1) return 0;
    return (((size_t)B * Hq * S * (D + 2) * 4 + 255) & ~(size_t)255) + (((size_t)B * Hq * 4 + 255) & ~(size_t)255);
}

inline int gqa_decode(int, const va_bufs*, const int*, int, int, int, int, int, int, void*, size_t, void*) {
    return VA_ERR_UNSUPPORTED;
}

}  // namespace va
