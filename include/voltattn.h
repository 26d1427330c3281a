/*
 * voltattn_b200 — C ABI of the B200 (sm_100a) fused dequant + online-softmax
 * attention decode path.
 *
 * The reference (kamilch1k/voltattn, one CUDA C++ file src/voltattn.cu) has no
 * library or FFI; its host interface is the internal C++ surface this header
 * replaces entry by entry (citations are src/voltattn.cu:line):
 *
 *   enum class Fmt / fmt_name            :676-686  -> va_fmt, va_fmt_name, va_fmt_from_name
 *   struct DeviceBufs                    :796-801  -> va_bufs (+ explicit workspace argument)
 *   launch(Fmt, DeviceBufs, H, L, D, S)  :803-835  -> va_decode
 *   combine<<<H,128>>>                   :651-672  -> va_combine_partials
 *   quantize(x, H, L, D, bits)           :705-745  -> va_quantize (a GPU kernel, bit-exact)
 *   probe_ceiling()                      :935-957  -> va_probe_ceiling
 *   CUDA_CHECK -> exit(1)                :49-58    -> status codes, va_status_string
 *
 * Conventions: every entry point returns a va_status (0 = success) and never
 * exits the process. Pointers are device pointers owned by the caller unless
 * stated otherwise. `stream` is a cudaStream_t passed as void* (NULL = the
 * legacy default stream, as the reference uses). Launches are asynchronous
 * with respect to the host, like the reference's launch().
 *
 * Data layout (identical to the reference, src/voltattn.cu:189, :254, :494,
 * :563, :694-703): K and V are head-major [H][L][D] rows.
 *   f16 formats : __half [H][L][D]
 *   q8          : int8   [H][L][D], code v in [-127,127]
 *   q4          : uint8  [H][L][D/2], byte k holds dims 2k (low nibble) and
 *                 2k+1 (high nibble), nibble = v + 8, v in [-7,7]
 *   q3          : uint8  [H][L][3D/8], element e of a row-major tensor sits at
 *                 bits 3*(e%8) of the little-endian 3-byte granule e/8, field = v+4
 *   scales      : __half [H][L][D/64] symmetric per-group scales (group = 64
 *                 consecutive dims), absent (NULL) for the f16 formats
 *   q, out      : __half [H][D]
 * D must be 64 or 128. K, V, scK, scV must be 16-byte aligned (cudaMalloc
 * and the torch allocator give 256).
 */
#ifndef VOLTATTN_B200_H
#define VOLTATTN_B200_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

#if defined(__GNUC__)
#define VA_API __attribute__((visibility("default")))
#else
#define VA_API
#endif

/* Formats, in the reference's order (src/voltattn.cu:676). The "+" formats run
 * the staged streaming kernels; f16 / q8 / q4 run the plain one-warp-per-position
 * kernel family kept as attribution baselines. bf16+ and f8+ have no reference
 * counterpart: bf16 rows (no scales), and e4m3 fp8 codes with fp16 scales per
 * 64-element group (va_quantize_f8). q4c+ (no counterpart either): q4 codes
 * with K scales per (head, channel) over all positions, scK = __half [H][D]
 * (va_quantize_kchan), and V scales per row, scV = __half [H][L]
 * (va_quantize_vtok); batch-1 decode at D = 128 with a fused workspace. */
typedef enum va_fmt {
    VA_F16 = 0,
    VA_F16P = 1,
    VA_Q8 = 2,
    VA_Q8P = 3,
    VA_Q4 = 4,
    VA_Q4P = 5,
    VA_Q3P = 6,
    VA_BF16P = 7,
    VA_F8P = 8,
    VA_Q4CP = 9
} va_fmt;

typedef enum va_status {
    VA_OK = 0,
    VA_ERR_INVALID = 1,     /* bad format, shape or null pointer */
    VA_ERR_ALIGN = 2,       /* a K/V/scale pointer is not 16-byte aligned */
    VA_ERR_WORKSPACE = 3,   /* workspace missing or smaller than required */
    VA_ERR_CUDA = 4,        /* a CUDA runtime call failed (see va_last_cuda_error) */
    VA_ERR_UNSUPPORTED = 5, /* D or format not supported by this build */
    VA_ERR_DEVICE = 6,      /* a kernel reported a device-side error (va_device_error) */
    VA_ERR_TOO_LARGE = 7    /* size beyond a stated maximum */
} va_status;

/* DeviceBufs (src/voltattn.cu:796-801) without `ws`, which every entry point
 * takes explicitly together with its size. */
typedef struct va_bufs {
    const void* K;
    const void* V;
    const void* scK; /* NULL for f16 formats */
    const void* scV; /* NULL for f16 formats */
    const void* q;   /* __half [H][D] */
    void* out;       /* __half [H][D] */
} va_bufs;

/* Library version as 10000*major + 100*minor + patch. No reference counterpart. */
VA_API int va_version(void);

/* fmt_name (src/voltattn.cu:677-686): "f16", "f16+", "q8", "q8+", "q4", "q4+",
 * "q3+" (without the reference's padding blanks); NULL for an invalid value. */
VA_API const char* va_fmt_name(int fmt);
/* Inverse of va_fmt_name; -1 when unknown. */
VA_API int va_fmt_from_name(const char* name);
/* Quantization bits of a format: 16, 8, 4 or 3 (qbits, src/voltattn.cu:691). */
VA_API int va_fmt_bits(int fmt);
/* Payload bytes of n elements (qbytes, src/voltattn.cu:692; 2n for f16). */
VA_API size_t va_payload_bytes(int fmt, size_t n);
/* Human-readable text of a va_status. */
VA_API const char* va_status_string(int status);
/* The cudaError_t of the last failing CUDA call made by this library on the
 * calling thread (0 if none). */
VA_API int va_last_cuda_error(void);

/* Workspace bytes va_decode needs for (H, D, S): the reference's H*S*(D+2)
 * floats of split partials (src/voltattn.cu:888) followed by one completion
 * counter per head. The counters must be zero before the first call (allocate
 * with cudaMemset / torch.zeros or call va_workspace_init); every completed
 * call leaves them zero again, so one workspace serves any number of calls
 * issued in order on one stream. */
VA_API size_t va_workspace_bytes(int H, int D, int S);
/* Zeroes a workspace of `bytes` bytes on `stream`. */
VA_API int va_workspace_init(void* ws, size_t bytes, void* stream);

/* A split count S for (fmt, H, L, D) that balances the persistent grid of the
 * current device (whole waves of work units); the reference's bench rule
 * (src/voltattn.cu:1026) is tuned for an 80-SM V100. Writes *S. */
VA_API int va_suggest_splits(int fmt, int H, int L, int D, int* S);

/* One batch-1 decode step over all H heads (launch, src/voltattn.cu:803-835):
 *   out[h] = softmax_j(q[h] . K[h][j] / sqrt(D)) . V[h][j]   (fp16 out, fp32 math)
 * with K/V dequantized in registers. S = number of KV-length splits per head
 * (1 <= S <= 65535); positions of head h are split into S contiguous ranges,
 * each producing an (m, l, o) partial merged by a log-sum-exp combine.
 * ws_bytes >= va_workspace_bytes(H, D, S): one launch, the combine fused into
 * the last CTA of each head. ws_bytes >= H*S*(D+2)*4 only (the reference's
 * workspace size): two launches, decode then combine. */
VA_API int va_decode(int fmt, const va_bufs* bufs, int H, int L, int D, int S, void* ws, size_t ws_bytes,
                     void* stream);

/* Split-L building block for multi-GPU decode (no reference counterpart; the
 * reference is single-GPU). As va_decode, but instead of fp16 output writes
 * each head's merged partial to `partial` = float [H][D+2] laid out like a
 * reference workspace slot (src/voltattn.cu:92-93): m (max scaled score, natural
 * log units), l (sum of exp(score - m)), o[D] (sum of exp(score - m) * V).
 * Requires ws_bytes >= va_workspace_bytes(H, D, S). */
VA_API int va_decode_partial(int fmt, const va_bufs* bufs, int H, int L, int D, int S, void* ws,
                             size_t ws_bytes, float* partial, void* stream);

/* Split-L exchange over NVLink peer memory, fused with the combine (no
 * reference counterpart). Each of R ranks (one GPU each) owns a buffer of
 * va_exchange_buffer_bytes(R, H, D) bytes, zeroed once, mapped into every
 * rank's address space (e.g. torch symmetric memory); `peer_buffers` is a
 * host array of the R buffers' device addresses as seen by this process
 * (peer_buffers[rank] is the local one). One call per decode step, with
 * epoch = 1, 2, 3, ... the same on all ranks: stores this rank's partial
 * (float [H][D+2], from va_decode_partial) into every rank's buffer as
 * 64-bit words tagged with the epoch, waits (bounded, ~1 s, then
 * va_device_error) until every word of the R ranks' partials carries the
 * epoch, and writes the merged fp16 output [H][D]. R <= 8. */
VA_API size_t va_exchange_buffer_bytes(int R, int H, int D);
VA_API int va_exchange_combine(const float* partial, int H, int D, int R, int rank, void* const* peer_buffers,
                               unsigned epoch, void* out, void* stream);

/* Split-L across GPUs in one launch per step (launch, src/voltattn.cu:803-835,
 * plus combine, :651-672, lifted across R GPUs): this rank decodes its range
 * [j0, j1) of every head's positions (K/V/scales of L = j1 - j0 rows per head,
 * layout as va_decode; S splits; fused workspace ws_bytes >=
 * va_workspace_bytes(H, D, S)), and the CTA that completes head h exchanges
 * the head's partial with the other ranks through peer_buffers (as
 * va_exchange_combine: va_exchange_buffer_bytes(R, H, D) each, mapped into
 * this process, zeroed once; epoch = 1, 2, 3, ... the same on all ranks, or
 * epoch = 0 on every call: the library counts the steps in the buffer itself,
 * so a sequence of calls can be captured in a CUDA graph and replayed; do
 * not mix the two ways on one buffer) and writes the merged fp16 output
 * [H][D] on every rank. q3+/q4+/q8+ at D = 128
 * on the tile kernel; other formats return VA_ERR_UNSUPPORTED (use
 * va_decode_partial + va_exchange_combine). Waits are bounded (~1 s, then
 * va_device_error = peer wait). */
/* Wall-clock limit of the split-L waits for the peers' partials
 * (va_exchange_combine, va_decode_splitl) in later launches: default 1 s,
 * 0 < seconds <= 60. A wait that runs out leaves the head's output untouched
 * and sets va_device_error to the peer-wait code (4). No reference
 * counterpart (the reference is single-GPU and exits on CUDA errors,
 * src/voltattn.cu:49-58). */
VA_API int va_set_peer_wait_limit(double seconds);

VA_API int va_decode_splitl(int fmt, const va_bufs* bufs, int H, int L, int D, int S, void* ws, size_t ws_bytes,
                            int R, int rank, void* const* peer_buffers, unsigned epoch, void* stream);

/* Log-sum-exp merge (combine, src/voltattn.cu:651-672) of R*S slots per head:
 * slots = float [R][H][S][D+2] (R = 1 is the reference's workspace layout; R > 1
 * is R gathered va_decode_partial / workspace blocks, e.g. one per GPU).
 * Writes fp16 out [H][D]. */
VA_API int va_combine_partials(const float* slots, int R, int H, int S, int D, void* out, void* stream);

/* Symmetric per-group quantizer (quantize, src/voltattn.cu:705-745) as a GPU
 * kernel, bit-exact with the reference's host function: for every 64-element
 * group of x (fp32 [H][L][D]) s = amax/lim (lim 127/7/3 for bits 8/4/3) is
 * rounded to fp16, and each code is round-half-even(x / stored scale) clamped
 * to [-lim, lim], packed as in the layout above. codes: va_payload_bytes
 * bytes; scales: __half [H][L][D/64]. x must be 16-byte aligned. */
VA_API int va_quantize(int bits, const float* x, void* codes, void* scales, int H, int L, int D,
                       void* stream);

/* fp8 group quantizer for f8+ (no reference counterpart), the rule of
 * va_quantize with lim = 448, the largest finite e4m3 value: per 64-element
 * group s = amax > 0 ? amax / 448 : 1 rounded to fp16, each code the e4m3
 * value of x / (stored s) rounded to nearest even with saturation to +-448
 * (nan stays nan). codes: 1 byte per element; scales: __half [H][L][D/64]. */
VA_API int va_quantize_f8(const float* x, void* codes, void* scales, int H, int L, int D, void* stream);

/* q4c+ quantizers (bits = 8 or 4), the rule of va_quantize with other groups:
 * va_quantize_kchan: per (head, channel) over the head's L positions,
 * scales = __half [H][D]; va_quantize_vtok: per row, scales = __half [H][L].
 * x = fp32 [H][L][D], 16-byte aligned; codes packed as q8 / q4. */
VA_API int va_quantize_kchan(int bits, const float* x, void* codes, void* scales, int H, int L, int D,
                             void* stream);
VA_API int va_quantize_vtok(int bits, const float* x, void* codes, void* scales, int H, int L, int D,
                            void* stream);

/* Copies `bytes` (a multiple of 16; both pointers 16-byte aligned) with a small
 * kernel of loads and stores. Either pointer may be pinned host memory
 * (cudaHostAlloc / cudaMallocHost: mapped into the device address space under
 * unified addressing), which moves a decode step's query in and its output
 * out without a copy-engine transfer (no reference counterpart). */
VA_API int va_copy_small(void* dst, const void* src, size_t bytes, void* stream);

/* One decode step with the query and the output in pinned host memory (no
 * reference counterpart; the reference's launch takes device buffers only):
 * copies q_host [H][D] fp16 into bufs->q, runs va_decode with its output
 * stored straight into out_host (bufs->out is not used), and returns once
 * out_host holds the result (it synchronizes the stream). Arguments as for va_decode;
 * q_host, out_host and bufs->q 16-byte aligned; q_host and out_host pinned
 * and mapped (pageable memory returns VA_ERR_INVALID). On a created stream
 * the launches are captured into a CUDA graph on the first call with a given
 * argument set and replayed on later calls with the same set (up to 16 sets
 * cached, oldest dropped; the pointers are validated when the set is first
 * seen). The first call therefore captures: make it outside any other stream
 * capture. On the legacy default stream (stream = NULL) the launches are
 * made directly. */
VA_API int va_decode_host(int fmt, const va_bufs* bufs, const void* q_host, void* out_host, int H, int L, int D,
                          int S, void* ws, size_t ws_bytes, void* stream);

/* KV append for decode loops (no reference counterpart; the reference
 * quantizes a whole cache once). Quantizes one new row per KV head of each
 * sequence, x = fp32 [B][Hkv][D], into a cache laid out as for
 * va_decode_gqa ([B][Hkv][Lcap] rows), at row pos[b] (device int32 [B]) of
 * every KV head of sequence b, with exactly the arithmetic of va_quantize:
 * appending rows one at a time produces the same bytes as quantizing the
 * whole cache at once. bits = 8 / 4 / 3 (codes + fp16 scales) or 16 (fp16
 * rows, scales unused). Rows with pos[b] outside [0, Lcap) are skipped. The
 * caller advances its lengths (e.g. lens += 1) for the next decode. */
VA_API int va_append_kv(int bits, const float* x, void* codes, void* scales, int B, int Hkv, int Lcap, int D,
                        const int* pos, void* stream);

/* Prefill: attention of Lq new tokens of one sequence over its cache (no
 * reference counterpart; the reference decodes one token at a time). The
 * tokens' K/V rows are already in the cache as its last Lq rows: K/V
 * [Hkv][L] rows in any format (scales [Hkv][L][D/64]; q4c+: K channel scales
 * [Hkv][D], V row scales [Hkv][L]). Token i (0 <= i < Lq) of query head h
 * attends to rows [0, L - Lq + i] of KV head h / (Hq/Hkv). q, out: __half
 * [Hq][Lq][D], 16-byte aligned. D = 128 (else VA_ERR_UNSUPPORTED). Runs on the tcgen05 tensor cores with the
 * cache dequantized to fp16 tile by tile. */
VA_API int va_prefill(int fmt, const va_bufs* bufs, int Hq, int Hkv, int L, int Lq, int D, void* stream);

/* va_prefill over a paged cache (no reference counterpart): the sequence's L
 * rows (its last Lq the new tokens) live in the pool of va_decode_paged, row j
 * of KV head k in page block_table[j / page_rows] (device int32 [max_pages],
 * max_pages * page_rows >= L) at row j % page_rows of
 * [num_pages][Hkv][page_rows] (scales alike). Entries outside [0, num_pages)
 * read page 0. Any page_rows >= 1. Formats as va_prefill except q4c+
 * (VA_ERR_UNSUPPORTED). */
VA_API int va_prefill_paged(int fmt, const va_bufs* bufs, const int* block_table, int max_pages, int page_rows,
                            int num_pages, int Hq, int Hkv, int L, int Lq, int D, void* stream);

/* va_prefill / va_prefill_paged with a workspace (no reference counterpart):
 * the cache rows [0, L) of every KV head are first converted once to fp16 in
 * ws (the same values the kernel above makes per block), then the attention
 * moves K/V tiles by tensor copies instead of converting them in every CTA
 * that reads them. ws: 16-byte aligned, ws_bytes >= va_prefill_workspace_bytes
 * (2 * Hkv * L rounded up to 128 * D * 2 bytes); its contents need no
 * initialisation. Same formats, shapes and results as va_prefill. */
VA_API size_t va_prefill_workspace_bytes(int Hkv, int L, int D);
VA_API int va_prefill_ws(int fmt, const va_bufs* bufs, int Hq, int Hkv, int L, int Lq, int D, void* ws,
                         size_t ws_bytes, void* stream);
VA_API int va_prefill_paged_ws(int fmt, const va_bufs* bufs, const int* block_table, int max_pages, int page_rows,
                               int num_pages, int Hq, int Hkv, int L, int Lq, int D, void* ws, size_t ws_bytes,
                               void* stream);

/* Multi-query decode (no reference counterpart), e.g. verifying Q speculative
 * tokens: the Q new tokens of each sequence are already appended to the cache
 * ([B][Hkv][Lmax] rows as for va_decode_gqa, lens[b] counting them), and
 * token i (0 <= i < Q) of query head h attends to rows [0, lens[b] - (Q-1-i))
 * of KV head h / (Hq/Hkv): causal among the new tokens. q, out: __half
 * [B][Hq][Q][D]. Every KV row is streamed once for all (Hq/Hkv) * Q query
 * slots, which must number 2, 4 or 8; q4+, D = 128 (else VA_ERR_UNSUPPORTED);
 * q 16-byte aligned; lens[b] >= Q. ws_bytes >= va_gqa_workspace_bytes(B,
 * Hq * Q, D, S). */
VA_API int va_decode_multiquery(int fmt, const va_bufs* bufs, const int* lens, int B, int Hq, int Hkv, int Q,
                                int Lmax, int D, int S, void* ws, size_t ws_bytes, void* stream);

/* Paged-cache forms of va_decode_gqa and va_append_kv (no reference
 * counterpart). The cache is a pool of num_pages pages; a page holds
 * page_rows rows of each of the Hkv KV heads: K/V [num_pages][Hkv][page_rows]
 * rows in format fmt, scales [num_pages][Hkv][page_rows][D/64]. Row j of KV
 * head k of sequence b lives in page block_table[b * max_pages + j / page_rows]
 * (device int32 [B][max_pages]) at row j % page_rows. lens: device int32 [B],
 * 1 <= lens[b] <= max_pages * page_rows. Entries outside [0, num_pages) read
 * page 0 (decode) or skip the row (append). Decode supports every "+" format
 * at D = 64 or 128 with Hq / Hkv in {1, 2, 4, 8} and page_rows a multiple of
 * 8, and q4c+ with Hq == Hkv at D = 128 (its V row scales paged like the
 * rows, its K channel scales [B][Hkv][D] per sequence, not paged): q3+ / q4+
 * / q8+ / q4c+ with Hq == Hkv and q4+ with Hq == 2, 4 or 8 * Hkv at D = 128
 * with page_rows a multiple of 32 run the tensor-core tile
 * kernels (splits s of a sequence take its 256-row tiles s, s + S, s + 2S,
 * ...); the rest the streaming / grouped-query kernels, which copy each run
 * of rows inside one page. Other shapes return VA_ERR_UNSUPPORTED. q must be
 * 16-byte aligned. ws as for va_decode_gqa (va_gqa_workspace_bytes). */
VA_API int va_decode_paged(int fmt, const va_bufs* bufs, const int* block_table, int max_pages, const int* lens,
                           int B, int Hq, int Hkv, int page_rows, int num_pages, int D, int S, void* ws,
                           size_t ws_bytes, void* stream);
/* Appends x = fp32 [B][Hkv][D] at logical row pos[b] of each sequence of a
 * paged cache, with the arithmetic of va_quantize (bits 16 / 8 / 4 / 3). */
VA_API int va_append_kv_paged(int bits, const float* x, void* codes, void* scales, const int* block_table,
                              int max_pages, int B, int Hkv, int page_rows, int num_pages, int D, const int* pos,
                              void* stream);

/* Read-bandwidth ceiling of `device` (probe_ceiling, src/voltattn.cu:935-957),
 * re-derived for HBM3e: streams a `bytes`-byte buffer (0 = 4 GiB) `reps` times
 * (0 = 20) after 3 warm-up passes with each of two kernels (wide vector loads;
 * bulk asynchronous copies into shared memory) and writes the best GB/s
 * (1e9 bytes/s) to *gbs. Allocates and frees its own buffer. Synchronous. */
VA_API int va_probe_ceiling(int device, size_t bytes, int reps, double* gbs);
/* The same for one method (0 = vector loads, 1 = bulk copies); *gbs = best. */
VA_API int va_probe_ceiling_method(int device, int method, size_t bytes, int reps, double* gbs);

/* Batched grouped-query decode with per-sequence lengths (no reference
 * counterpart; the reference is batch 1, one KV head per query head).
 * K/V: [B][Hkv][Lmax][D] rows in format fmt (rows >= lens[b] are never read),
 * scales [B][Hkv][Lmax][D/64]; q, out: __half [B][Hq][D]; lens: device int32
 * [B], 1 <= lens[b] <= Lmax. Query head hq reads KV head hq / (Hq / Hkv).
 * Each (sequence, KV head) streams its cache once for all of its query heads
 * (G = Hq/Hkv in {1, 2, 4, 8}; "+" formats only). S = splits per sequence:
 * positions [s*c, (s+1)*c) with c = Lmax/S rounded up to 8 (splits past
 * lens[b] are empty). ws_bytes >= va_gqa_workspace_bytes(B, Hq, D, S), zeroed
 * before first use like va_decode's workspace. q4c+: Hq == Hkv and D = 128,
 * K channel scales [B][Hkv][D] (va_quantize_kchan with H = B*Hkv, L = Lmax),
 * V row scales [B][Hkv][Lmax], q 16-byte aligned. */
VA_API size_t va_gqa_workspace_bytes(int B, int Hq, int D, int S);
VA_API int va_decode_gqa(int fmt, const va_bufs* bufs, const int* lens, int B, int Hq, int Hkv, int Lmax,
                         int D, int S, void* ws, size_t ws_bytes, void* stream);

/* va_decode for callers that cannot allocate device memory. No counterpart in
 * the reference. Some hosts of this library cannot call cudaMalloc: code
 * running inside a CUDA-graph-building framework that forbids allocation
 * between captures, plugins whose host owns the whole memory pool, and
 * callers that keep device memory fixed after start-up. This entry point takes
 * the same inputs and outputs as va_decode but no workspace. The workspace is
 * a fixed 4 MiB array built into the library: every GPU that loads the
 * library holds it until the process exits. The required size is
 * va_workspace_bytes(H, D, S); calls that need more than 4 MiB return
 * VA_ERR_TOO_LARGE before launching anything. The first call on a device looks
 * up the array's device address (once per device, with that device current),
 * so make that first call before any stream capture begins. Every call
 * shares the one array: each call clears its completion counters on `stream`
 * first, and calls whose kernels overlap on the GPU (different streams, or
 * different host threads) race on it and must be serialised by the caller.
 * Allocates nothing (no cudaMalloc, no cudaFree). */
VA_API int va_decode_noalloc(int fmt, const va_bufs* bufs, int H, int L, int D, int S, void* stream);

/* Device-side error word (bounded waits that gave up, etc.). Reads and clears
 * the flag of the current device; *code = 0 when no kernel reported one. */
VA_API int va_device_error(int* code);

#ifdef __cplusplus
} /* extern "C" */
#endif

#endif /* VOLTATTN_B200_H */
