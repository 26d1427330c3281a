// voltattn_b200 — C++ mirror of the reference's host interface, over the C ABI
// in voltattn.h. Same names and argument meaning as src/voltattn.cu:
//   enum class Fmt            :676      fmt_name  :677-686
//   struct DeviceBufs         :796-801  launch()  :803-835
//   qbits / qbytes            :691-692  GROUP     :60
// so host code written against the reference compiles against this header.
// Error behaviour: the reference's CUDA_CHECK prints and exit(1)s
// (src/voltattn.cu:49-58); here every failure throws voltattn::Error carrying
// the va_status, which a caller can turn into the same exit.
#pragma once

#include <cuda_fp16.h>

#include <cstddef>
#include <stdexcept>
#include <string>

#include "voltattn.h"

namespace voltattn {

constexpr int GROUP = 64;

enum class Fmt { F16, F16M, Q8, Q8M, Q4, Q4M, Q3M };

struct Error : std::runtime_error {
    int status;
    Error(int st, const std::string& what)
        : std::runtime_error(what + ": " + va_status_string(st)), status(st) {}
};

inline void check(int st, const char* what) {
    if (st != VA_OK) throw Error(st, what);
}

inline const char* fmt_name(Fmt f) { return va_fmt_name(static_cast<int>(f)); }
inline bool is_q4(Fmt f) { return f == Fmt::Q4 || f == Fmt::Q4M; }
inline bool is_q3(Fmt f) { return f == Fmt::Q3M; }
inline bool is_f16(Fmt f) { return f == Fmt::F16 || f == Fmt::F16M; }
inline int qbits(Fmt f) { return is_q3(f) ? 3 : is_q4(f) ? 4 : 8; }
inline size_t qbytes(int bits, size_t n) { return bits == 8 ? n : bits == 4 ? n / 2 : n * 3 / 8; }

// The reference's DeviceBufs: caller-owned device buffers; ws holds
// H*S*(D+2) floats (src/voltattn.cu:888).
struct DeviceBufs {
    void *K = nullptr, *V = nullptr, *scK = nullptr, *scV = nullptr;
    __half* q = nullptr;
    __half* out = nullptr;
    float* ws = nullptr;
};

// launch(): enqueues one decode on the default stream. With the reference's
// workspace size it runs the decode then the combine (two launches, as the
// reference); pass a larger workspace through voltattn::decode for the fused
// single launch.
inline void launch(Fmt f, const DeviceBufs& b, int H, int L, int D, int S, cudaStream_t stream = nullptr) {
    const va_bufs vb{b.K, b.V, b.scK, b.scV, b.q, b.out};
    check(va_decode(static_cast<int>(f), &vb, H, L, D, S, b.ws, (size_t)H * S * (D + 2) * sizeof(float), stream),
          "voltattn::launch");
}

// Fused single-launch decode with a workspace of workspace_bytes(H, D, S).
inline size_t workspace_bytes(int H, int D, int S) { return va_workspace_bytes(H, D, S); }
inline void decode(Fmt f, const DeviceBufs& b, int H, int L, int D, int S, void* ws, size_t ws_bytes,
                   cudaStream_t stream = nullptr) {
    const va_bufs vb{b.K, b.V, b.scK, b.scV, b.q, b.out};
    check(va_decode(static_cast<int>(f), &vb, H, L, D, S, ws, ws_bytes, stream), "voltattn::decode");
}

// quantize() on the GPU: x fp32 [H][L][D] -> packed codes + fp16 scales.
inline void quantize(const float* x, int H, int L, int D, int bits, void* codes, __half* scales,
                     cudaStream_t stream = nullptr) {
    check(va_quantize(bits, x, codes, scales, H, L, D, stream), "voltattn::quantize");
}

// probe_ceiling(): GB/s of the current device's read ceiling.
inline double probe_ceiling(int device = 0) {
    double g = 0.0;
    check(va_probe_ceiling(device, 0, 0, &g), "voltattn::probe_ceiling");
    return g;
}

}  // namespace voltattn
