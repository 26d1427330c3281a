"""voltattn_b200 — B200-native fused dequant + online-softmax attention decode.

Python mirror of the reference's host interface (kamilch1k/voltattn,
src/voltattn.cu) over the C ABI in include/voltattn.h, loaded with ctypes from
the in-tree libvoltattn_b200.so. Device memory, streams and
torch.distributed come from PyTorch; all compute runs in this package's CUDA
kernels. There is no CPU fallback: importing the package fails loudly when the
shared library is missing.

Reference names kept: `Fmt` (:676), `fmt_name` (:677), `DeviceBufs` (:796),
`launch` (:803), `quantize` (:709), `probe_ceiling` (:935), `GROUP` (:60),
`qbits` / `qbytes` (:691-692).
"""
from __future__ import annotations

import ctypes as C
import enum
import os
from dataclasses import dataclass
from typing import Optional

_HERE = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(_HERE, "libvoltattn_b200.so")

GROUP = 64


class VoltAttnError(RuntimeError):
    def __init__(self, status: int, what: str):
        self.status = status
        super().__init__(f"{what}: {_lib.va_status_string(status).decode()} (status {status}"
                         + (f", cudaError {_lib.va_last_cuda_error()}" if status == 4 else "") + ")")


def _load():
    if not os.path.exists(LIB_PATH):
        raise ImportError(f"voltattn_b200: {LIB_PATH} is missing — build it with `make` or "
                          "`python -c 'import __graft_entry__ as g; g.build()'` (no CPU fallback exists)")
    lib = C.CDLL(LIB_PATH)
    vp, i, sz = C.c_void_p, C.c_int, C.c_size_t
    lib.va_version.restype = i
    lib.va_fmt_name.argtypes = [i]; lib.va_fmt_name.restype = C.c_char_p
    lib.va_fmt_from_name.argtypes = [C.c_char_p]; lib.va_fmt_from_name.restype = i
    lib.va_fmt_bits.argtypes = [i]; lib.va_fmt_bits.restype = i
    lib.va_payload_bytes.argtypes = [i, sz]; lib.va_payload_bytes.restype = sz
    lib.va_status_string.argtypes = [i]; lib.va_status_string.restype = C.c_char_p
    lib.va_last_cuda_error.restype = i
    lib.va_workspace_bytes.argtypes = [i, i, i]; lib.va_workspace_bytes.restype = sz
    lib.va_workspace_init.argtypes = [vp, sz, vp]; lib.va_workspace_init.restype = i
    lib.va_suggest_splits.argtypes = [i, i, i, i, C.POINTER(i)]; lib.va_suggest_splits.restype = i
    lib.va_decode.argtypes = [i, C.POINTER(VaBufs), i, i, i, i, vp, sz, vp]; lib.va_decode.restype = i
    lib.va_decode_partial.argtypes = [i, C.POINTER(VaBufs), i, i, i, i, vp, sz, vp, vp]
    lib.va_decode_partial.restype = i
    lib.va_combine_partials.argtypes = [vp, i, i, i, i, vp, vp]; lib.va_combine_partials.restype = i
    lib.va_quantize.argtypes = [i, vp, vp, vp, i, i, i, vp]; lib.va_quantize.restype = i
    lib.va_probe_ceiling.argtypes = [i, sz, i, C.POINTER(C.c_double)]; lib.va_probe_ceiling.restype = i
    lib.va_probe_ceiling_method.argtypes = [i, i, sz, i, C.POINTER(C.c_double)]
    lib.va_probe_ceiling_method.restype = i
    lib.va_gqa_workspace_bytes.argtypes = [i, i, i, i]; lib.va_gqa_workspace_bytes.restype = sz
    lib.va_decode_gqa.argtypes = [i, C.POINTER(VaBufs), vp, i, i, i, i, i, i, vp, sz, vp]
    lib.va_decode_gqa.restype = i
    lib.va_decode_noalloc.argtypes = [i, C.POINTER(VaBufs), i, i, i, i, vp]; lib.va_decode_noalloc.restype = i
    lib.va_exchange_buffer_bytes.argtypes = [i, i, i]; lib.va_exchange_buffer_bytes.restype = sz
    lib.va_exchange_combine.argtypes = [vp, i, i, i, i, C.POINTER(C.c_void_p), C.c_uint, vp, vp]
    lib.va_exchange_combine.restype = i
    lib.va_decode_splitl.argtypes = [i, C.POINTER(VaBufs), i, i, i, i, vp, sz, i, i, C.POINTER(C.c_void_p), C.c_uint,
                                     vp]
    lib.va_decode_splitl.restype = i
    lib.va_set_peer_wait_limit.argtypes = [C.c_double]; lib.va_set_peer_wait_limit.restype = i
    lib.va_append_kv.argtypes = [i, vp, vp, vp, i, i, i, i, vp, vp]; lib.va_append_kv.restype = i
    lib.va_quantize_f8.argtypes = [vp, vp, vp, i, i, i, vp]; lib.va_quantize_f8.restype = i
    lib.va_copy_small.argtypes = [vp, vp, sz, vp]; lib.va_copy_small.restype = i
    lib.va_decode_host.argtypes = [i, C.POINTER(VaBufs), vp, vp, i, i, i, i, vp, sz, vp]
    lib.va_decode_host.restype = i
    for fn in ("va_quantize_kchan", "va_quantize_vtok"):
        getattr(lib, fn).argtypes = [i, vp, vp, vp, i, i, i, vp]
        getattr(lib, fn).restype = i
    lib.va_decode_multiquery.argtypes = [i, C.POINTER(VaBufs), vp, i, i, i, i, i, i, i, vp, sz, vp]
    lib.va_decode_multiquery.restype = i
    lib.va_prefill.argtypes = [i, C.POINTER(VaBufs), i, i, i, i, i, vp]
    lib.va_prefill.restype = i
    lib.va_prefill_workspace_bytes.argtypes = [i, i, i]; lib.va_prefill_workspace_bytes.restype = sz
    lib.va_prefill_ws.argtypes = [i, C.POINTER(VaBufs), i, i, i, i, i, vp, sz, vp]
    lib.va_prefill_ws.restype = i
    lib.va_prefill_paged_ws.argtypes = [i, C.POINTER(VaBufs), vp, i, i, i, i, i, i, i, i, vp, sz, vp]
    lib.va_prefill_paged_ws.restype = i
    lib.va_prefill_paged.argtypes = [i, C.POINTER(VaBufs), vp, i, i, i, i, i, i, i, i, vp]
    lib.va_prefill_paged.restype = i
    lib.va_decode_paged.argtypes = [i, C.POINTER(VaBufs), vp, i, vp, i, i, i, i, i, i, i, vp, sz, vp]
    lib.va_decode_paged.restype = i
    lib.va_append_kv_paged.argtypes = [i, vp, vp, vp, vp, i, i, i, i, i, i, vp, vp]
    lib.va_append_kv_paged.restype = i
    lib.va_device_error.argtypes = [C.POINTER(i)]; lib.va_device_error.restype = i
    return lib


class VaBufs(C.Structure):
    _fields_ = [("K", C.c_void_p), ("V", C.c_void_p), ("scK", C.c_void_p), ("scV", C.c_void_p),
                ("q", C.c_void_p), ("out", C.c_void_p)]


_lib = _load()


def lib():
    """The loaded ctypes library (for tests that call the C ABI directly)."""
    return _lib


def _check(status: int, what: str):
    if status != 0:
        raise VoltAttnError(status, what)


class Fmt(enum.IntEnum):
    """Formats in the reference's order (src/voltattn.cu:676)."""
    F16 = 0
    F16M = 1
    Q8 = 2
    Q8M = 3
    Q4 = 4
    Q4M = 5
    Q3M = 6
    BF16M = 7  # bf16+ (no reference counterpart)
    F8M = 8    # f8+: e4m3 codes with fp16 group scales (no reference counterpart)
    Q4CM = 9   # q4c+: q4 codes, K scales per (head, channel), V scales per row (no reference counterpart)

    @property
    def name_str(self) -> str:
        return fmt_name(self)

    @classmethod
    def parse(cls, f) -> "Fmt":
        if isinstance(f, Fmt):
            return f
        if isinstance(f, int):
            return cls(f)
        v = _lib.va_fmt_from_name(str(f).strip().encode())
        if v < 0:
            raise ValueError(f"unknown format {f!r}")
        return cls(v)


FORMATS = [Fmt(i) for i in range(7)]  # the reference's formats
EXTRA_FORMATS = [Fmt.BF16M, Fmt.F8M, Fmt.Q4CM]


def fmt_name(f) -> str:
    return _lib.va_fmt_name(int(Fmt.parse(f))).decode()


def is_f16(f) -> bool:
    return Fmt.parse(f) in (Fmt.F16, Fmt.F16M)


def qbits(f) -> int:
    """Quantization bits of a quantized format (src/voltattn.cu:691)."""
    return {Fmt.Q8: 8, Fmt.Q8M: 8, Fmt.Q4: 4, Fmt.Q4M: 4, Fmt.Q3M: 3, Fmt.F8M: 8, Fmt.Q4CM: 4}.get(Fmt.parse(f), 8)


def qbytes(bits: int, n: int) -> int:
    """Payload bytes of n codes (src/voltattn.cu:692)."""
    return n if bits == 8 else n // 2 if bits == 4 else n * 3 // 8


def payload_bytes(f, n: int) -> int:
    return int(_lib.va_payload_bytes(int(Fmt.parse(f)), n))


def workspace_bytes(H: int, D: int, S: int) -> int:
    return int(_lib.va_workspace_bytes(H, D, S))


def suggest_splits(f, H: int, L: int, D: int) -> int:
    s = C.c_int(0)
    _check(_lib.va_suggest_splits(int(Fmt.parse(f)), H, L, D, C.byref(s)), "suggest_splits")
    return s.value


def _ptr(t) -> Optional[int]:
    return None if t is None else t.data_ptr()


def _stream_ptr(stream) -> Optional[int]:
    import torch
    if stream is None:
        stream = torch.cuda.current_stream()
    return stream.cuda_stream


@dataclass
class DeviceBufs:
    """The reference's DeviceBufs (src/voltattn.cu:796-801) over torch tensors:
    K, V codes (uint8 / int8 / float16), scK / scV fp16 group scales (None for
    the f16 formats), q and out fp16 [H][D], ws float32 workspace."""
    K: object
    V: object
    scK: object = None
    scV: object = None
    q: object = None
    out: object = None
    ws: object = None

    def va(self) -> VaBufs:
        return VaBufs(_ptr(self.K), _ptr(self.V), _ptr(self.scK), _ptr(self.scV), _ptr(self.q), _ptr(self.out))


def new_workspace(H: int, D: int, S: int, device=None):
    """A zeroed workspace for the fused single-launch decode."""
    import torch
    return torch.zeros(workspace_bytes(H, D, S), dtype=torch.uint8, device=device or "cuda")


def launch(fmt, b: DeviceBufs, H: int, L: int, D: int, S: int, stream=None):
    """One decode step (launch, src/voltattn.cu:803). With b.ws of
    workspace_bytes(H, D, S) bytes (zeroed once) the combine is fused into the
    decode launch; with the reference's H*S*(D+2) floats it runs as a second
    launch. Asynchronous on `stream` (default: torch's current stream)."""
    vb = b.va()
    _check(_lib.va_decode(int(Fmt.parse(fmt)), C.byref(vb), H, L, D, S, _ptr(b.ws),
                          b.ws.numel() * b.ws.element_size(), _stream_ptr(stream)), "launch")


def decode_partial(fmt, b: DeviceBufs, H: int, L: int, D: int, S: int, partial, stream=None):
    """Per-head merged (m, l, o[D]) partials, float32 [H][D+2] (split-L building block)."""
    vb = b.va()
    _check(_lib.va_decode_partial(int(Fmt.parse(fmt)), C.byref(vb), H, L, D, S, _ptr(b.ws),
                                  b.ws.numel() * b.ws.element_size(), _ptr(partial), _stream_ptr(stream)),
           "decode_partial")


def combine_partials(slots, R: int, H: int, S: int, D: int, out, stream=None):
    """Log-sum-exp merge of float32 slots [R][H][S][D+2] into fp16 out [H][D]."""
    _check(_lib.va_combine_partials(_ptr(slots), R, H, S, D, _ptr(out), _stream_ptr(stream)),
           "combine_partials")


def quantize(x, bits: int, H: int, L: int, D: int, codes=None, scales=None, stream=None):
    """GPU group quantizer (quantize, src/voltattn.cu:709), bit-exact with the
    reference. x: float32 CUDA tensor with H*L*D elements. Returns (codes uint8,
    scales float16)."""
    import torch
    n = H * L * D
    if x.dtype != torch.float32 or not x.is_cuda or x.numel() != n or not x.is_contiguous():
        raise ValueError("quantize: x must be a contiguous float32 CUDA tensor of H*L*D elements")
    if codes is None:
        codes = torch.empty(qbytes(bits, n), dtype=torch.uint8, device=x.device)
    if scales is None:
        scales = torch.empty(H * L * (D // GROUP), dtype=torch.float16, device=x.device)
    _check(_lib.va_quantize(bits, _ptr(x), _ptr(codes), _ptr(scales), H, L, D, _stream_ptr(stream)), "quantize")
    return codes, scales


def append_kv(x, bits: int, codes, scales, B: int, Hkv: int, Lcap: int, D: int, pos, stream=None):
    """Quantize one new row per KV head of each sequence (x fp32 [B][Hkv][D])
    into a [B][Hkv][Lcap] cache at row pos[b] (int32 CUDA tensor), bit-exact
    with quantize() of the whole cache. bits 16 stores fp16 rows."""
    _check(_lib.va_append_kv(bits, _ptr(x), _ptr(codes), _ptr(scales), B, Hkv, Lcap, D, _ptr(pos),
                             _stream_ptr(stream)), "append_kv")


def copy_small(dst, src, stream=None):
    """Copy between two same-size tensors by a small kernel; either may be pinned
    host memory (device-mapped under unified addressing)."""
    nbytes = src.numel() * src.element_size()
    assert dst.numel() * dst.element_size() == nbytes
    _check(_lib.va_copy_small(_ptr(dst), _ptr(src), nbytes, _stream_ptr(stream)), "copy_small")


def decode_host(fmt, b: DeviceBufs, q_host, out_host, H: int, L: int, D: int, S: int, stream=None):
    """One decode step with q and out in pinned host memory (va_decode_host):
    q_host -> b.q, decode, b.out -> out_host; returns once out_host holds the
    output. On a created stream the step is a cached CUDA graph after its first
    call with these arguments."""
    vb = b.va()
    _check(_lib.va_decode_host(int(Fmt.parse(fmt)), C.byref(vb), _ptr(q_host), _ptr(out_host), H, L, D, S,
                               _ptr(b.ws), b.ws.numel() * b.ws.element_size(), _stream_ptr(stream)), "decode_host")


class HostStep:
    """decode_host with its arguments bound once, for serving loops: calling
    the object runs one step (one C call; the tensors must stay alive and in
    place, as for the captured graph behind it)."""

    def __init__(self, fmt, b: DeviceBufs, q_host, out_host, H: int, L: int, D: int, S: int, stream=None):
        self._keep = (b, q_host, out_host, stream)
        self._vb = b.va()
        self._args = (int(Fmt.parse(fmt)), C.byref(self._vb), _ptr(q_host), _ptr(out_host), H, L, D, S,
                      _ptr(b.ws), b.ws.numel() * b.ws.element_size(), _stream_ptr(stream))
        self._fn = _lib.va_decode_host

    def __call__(self):
        rc = self._fn(*self._args)
        if rc:
            _check(rc, "decode_host")


def quantize_f8(x, H: int, L: int, D: int, codes=None, scales=None, stream=None):
    """GPU fp8 (e4m3) group quantizer for f8+: fp32 [H][L][D] -> 1-byte codes
    and fp16 scales [H][L][D/64] (allocated when not given)."""
    import torch
    if codes is None:
        codes = torch.empty(H * L * D, dtype=torch.uint8, device=x.device)
    if scales is None:
        scales = torch.empty(H * L * (D // 64), dtype=torch.float16, device=x.device)
    _check(_lib.va_quantize_f8(_ptr(x), _ptr(codes), _ptr(scales), H, L, D, _stream_ptr(stream)), "quantize_f8")
    return codes, scales


def quantize_kchan(x, bits: int, H: int, L: int, D: int, stream=None):
    """q4c+ K quantizer: scales per (head, channel) over all positions, [H][D]."""
    import torch
    codes = torch.empty(H * L * D * bits // 8, dtype=torch.uint8, device=x.device)
    scales = torch.empty(H * D, dtype=torch.float16, device=x.device)
    _check(_lib.va_quantize_kchan(bits, _ptr(x), _ptr(codes), _ptr(scales), H, L, D, _stream_ptr(stream)),
           "quantize_kchan")
    return codes, scales


def quantize_vtok(x, bits: int, H: int, L: int, D: int, stream=None):
    """q4c+ V quantizer: one scale per row, [H][L]."""
    import torch
    codes = torch.empty(H * L * D * bits // 8, dtype=torch.uint8, device=x.device)
    scales = torch.empty(H * L, dtype=torch.float16, device=x.device)
    _check(_lib.va_quantize_vtok(bits, _ptr(x), _ptr(codes), _ptr(scales), H, L, D, _stream_ptr(stream)),
           "quantize_vtok")
    return codes, scales


def append_kv_paged(x, bits: int, codes, scales, block_table, max_pages: int, B: int, Hkv: int, page_rows: int,
                    num_pages: int, D: int, pos, stream=None):
    """append_kv into a paged cache ([num_pages][Hkv][page_rows] rows; row j of
    sequence b in page block_table[b][j // page_rows])."""
    _check(_lib.va_append_kv_paged(bits, _ptr(x), _ptr(codes), _ptr(scales), _ptr(block_table), max_pages, B, Hkv,
                                   page_rows, num_pages, D, _ptr(pos), _stream_ptr(stream)), "append_kv_paged")


def decode_multiquery(fmt, b: DeviceBufs, lens, B: int, Hq: int, Hkv: int, Q: int, Lmax: int, D: int, S: int,
                      stream=None):
    """Q new tokens per sequence (already in the cache, counted in lens), each
    causal among the new tokens; q / out fp16 [B][Hq][Q][D]."""
    vb = b.va()
    _check(_lib.va_decode_multiquery(int(Fmt.parse(fmt)), C.byref(vb), _ptr(lens), B, Hq, Hkv, Q, Lmax, D, S,
                                     _ptr(b.ws), b.ws.numel() * b.ws.element_size(), _stream_ptr(stream)),
           "decode_multiquery")


def prefill_workspace_bytes(Hkv: int, L: int, D: int) -> int:
    return int(_lib.va_prefill_workspace_bytes(Hkv, L, D))


def _prefill_ws(b: DeviceBufs, Hkv: int, L: int, D: int, staged: bool):
    """The staging workspace: b.ws when it is large enough, else a new one;
    None for the unstaged kernel."""
    if not staged:
        return None
    need = prefill_workspace_bytes(Hkv, L, D)
    if b.ws is not None and b.ws.numel() * b.ws.element_size() >= need:
        return b.ws
    import torch
    return torch.empty(need, dtype=torch.uint8, device=b.q.device)


def prefill(fmt, b: DeviceBufs, Hq: int, Hkv: int, L: int, Lq: int, D: int, stream=None, staged: bool = True):
    """Attention of the Lq new tokens of one sequence over its cache (the
    tokens' rows are its last Lq rows; token i sees rows [0, L - Lq + i]) on
    the tcgen05 tensor cores. b.K / b.V: [Hkv][L] rows; b.q, b.out: fp16
    [Hq][Lq][D]. staged (default): the cache is converted once into a
    workspace (b.ws if large enough, else allocated) and the tiles move by
    tensor copies (va_prefill_ws); staged=False: va_prefill, no workspace."""
    vb = b.va()
    ws = _prefill_ws(b, Hkv, L, D, staged)
    if ws is None:
        _check(_lib.va_prefill(int(Fmt.parse(fmt)), C.byref(vb), Hq, Hkv, L, Lq, D, _stream_ptr(stream)), "prefill")
    else:
        _check(_lib.va_prefill_ws(int(Fmt.parse(fmt)), C.byref(vb), Hq, Hkv, L, Lq, D, _ptr(ws),
                                  ws.numel() * ws.element_size(), _stream_ptr(stream)), "prefill")


def prefill_paged(fmt, b: DeviceBufs, block_table, max_pages: int, page_rows: int, num_pages: int, Hq: int,
                  Hkv: int, L: int, Lq: int, D: int, stream=None, staged: bool = True):
    """prefill over a paged cache: b.K / b.V (and scales) are the page pool
    [num_pages][Hkv][page_rows], block_table int32 [max_pages] (CUDA)."""
    vb = b.va()
    ws = _prefill_ws(b, Hkv, L, D, staged)
    if ws is None:
        _check(_lib.va_prefill_paged(int(Fmt.parse(fmt)), C.byref(vb), _ptr(block_table), max_pages, page_rows,
                                     num_pages, Hq, Hkv, L, Lq, D, _stream_ptr(stream)), "prefill_paged")
    else:
        _check(_lib.va_prefill_paged_ws(int(Fmt.parse(fmt)), C.byref(vb), _ptr(block_table), max_pages, page_rows,
                                        num_pages, Hq, Hkv, L, Lq, D, _ptr(ws), ws.numel() * ws.element_size(),
                                        _stream_ptr(stream)), "prefill_paged")


def decode_paged(fmt, b: DeviceBufs, block_table, max_pages: int, lens, B: int, Hq: int, Hkv: int, page_rows: int,
                 num_pages: int, D: int, S: int, stream=None):
    """Grouped-query / batch decode over a paged cache (block_table int32
    [B][max_pages], lens int32 [B], CUDA tensors); workspace as decode_gqa."""
    vb = b.va()
    _check(_lib.va_decode_paged(int(Fmt.parse(fmt)), C.byref(vb), _ptr(block_table), max_pages, _ptr(lens), B, Hq,
                                Hkv, page_rows, num_pages, D, S, _ptr(b.ws), b.ws.numel() * b.ws.element_size(),
                                _stream_ptr(stream)), "decode_paged")


def probe_ceiling(device: int = 0, nbytes: int = 0, reps: int = 0, method: Optional[int] = None) -> float:
    """HBM read ceiling in GB/s (probe_ceiling, src/voltattn.cu:935)."""
    g = C.c_double(0.0)
    if method is None:
        _check(_lib.va_probe_ceiling(device, nbytes, reps, C.byref(g)), "probe_ceiling")
    else:
        _check(_lib.va_probe_ceiling_method(device, method, nbytes, reps, C.byref(g)), "probe_ceiling")
    return g.value


def gqa_workspace_bytes(B: int, Hq: int, D: int, S: int) -> int:
    return int(_lib.va_gqa_workspace_bytes(B, Hq, D, S))


def decode_gqa(fmt, b: DeviceBufs, lens, B: int, Hq: int, Hkv: int, Lmax: int, D: int, S: int, stream=None):
    """Batched grouped-query decode with per-sequence lengths (int32 CUDA tensor)."""
    vb = b.va()
    _check(_lib.va_decode_gqa(int(Fmt.parse(fmt)), C.byref(vb), _ptr(lens), B, Hq, Hkv, Lmax, D, S, _ptr(b.ws),
                              b.ws.numel() * b.ws.element_size(), _stream_ptr(stream)), "decode_gqa")


def exchange_buffer_bytes(R: int, H: int, D: int) -> int:
    return int(_lib.va_exchange_buffer_bytes(R, H, D))


def exchange_combine(partial, H: int, D: int, R: int, rank: int, peer_ptrs, epoch: int, out, stream=None):
    """Split-L exchange over peer memory fused with the combine (see
    include/voltattn.h, va_exchange_combine). peer_ptrs: R device addresses."""
    arr = (C.c_void_p * R)(*peer_ptrs)
    _check(_lib.va_exchange_combine(_ptr(partial), H, D, R, rank, arr, epoch, _ptr(out), _stream_ptr(stream)),
           "exchange_combine")


def decode_splitl(fmt, b: DeviceBufs, H: int, L: int, D: int, S: int, R: int, rank: int, peer_array, epoch: int,
                  stream=None):
    """Split-L step in one launch (include/voltattn.h, va_decode_splitl): this
    rank's L positions per head, exchanged and merged with the other ranks'
    into b.out. peer_array: a ctypes array of the R peer buffer addresses
    (built once by the caller)."""
    vb = b.va()
    _check(_lib.va_decode_splitl(int(Fmt.parse(fmt)), C.byref(vb), H, L, D, S, _ptr(b.ws),
                                 b.ws.numel() * b.ws.element_size(), R, rank, peer_array, epoch,
                                 _stream_ptr(stream)), "decode_splitl")


def set_peer_wait_limit(seconds: float) -> None:
    """Bound of the split-L waits for the peers' partials (default 1 s)."""
    _check(_lib.va_set_peer_wait_limit(float(seconds)), "set_peer_wait_limit")


def device_error() -> int:
    """Reads and clears the device error word (bounded waits that gave up)."""
    c = C.c_int(0)
    _check(_lib.va_device_error(C.byref(c)), "device_error")
    return c.value


def decode(fmt, K, V, scK, scV, q, H: int, L: int, D: int, S: Optional[int] = None, out=None, ws=None,
           stream=None):
    """Convenience: allocates out / workspace as needed and runs one decode."""
    import torch
    if S is None:
        S = suggest_splits(fmt, H, L, D)
    if out is None:
        out = torch.empty(H * D, dtype=torch.float16, device=q.device)
    if ws is None:
        ws = new_workspace(H, D, S, q.device)
    launch(fmt, DeviceBufs(K, V, scK, scV, q, out, ws), H, L, D, S, stream)
    return out
