"""ctypes bindings to the test-only checkers built by oracle/Makefile.

TEST INFRASTRUCTURE ONLY: imported by tests/, __graft_entry__.smoke() and the
cpu_baseline / reference legs of bench.py. The product package never imports
this module.

* `Oracle`  — liboracle.so, the CPU restatement of the reference's host path
  (src/voltattn.cu:705-794, :839-846, :959-965, :651-672).
* `RefLib`  — _ref/libvoltattn_ref.so, the reference translation unit itself
  compiled from its own source (present only where it was built).
"""
from __future__ import annotations

import ctypes as C
import os
import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
ORACLE_SO = os.path.join(HERE, "liboracle.so")
REF_SO = os.path.join(HERE, "_ref", "libvoltattn_ref.so")

GROUP = 64
BITS = {"q8": 8, "q8+": 8, "q4": 4, "q4+": 4, "q3+": 3}
FORMATS = ["f16", "f16+", "q8", "q8+", "q4", "q4+", "q3+"]  # src/voltattn.cu:676-686
SELFTEST_CASES = [  # (H, L, D, S), src/voltattn.cu:913-916
    (8, 257, 128, 1), (8, 257, 128, 3), (2, 4096, 128, 5),
    (40, 1000, 128, 2), (8, 129, 64, 1), (8, 513, 64, 4),
]

_f32p = np.ctypeslib.ndpointer(np.float32, flags="C_CONTIGUOUS")
_u16p = np.ctypeslib.ndpointer(np.uint16, flags="C_CONTIGUOUS")
_u8p = np.ctypeslib.ndpointer(np.uint8, flags="C_CONTIGUOUS")
_i32p = np.ctypeslib.ndpointer(np.int32, flags="C_CONTIGUOUS")


def payload_bytes(bits: int, n: int) -> int:
    return n if bits == 8 else n // 2 if bits == 4 else n * 3 // 8


class Oracle:
    def __init__(self, path: str = ORACLE_SO):
        if not os.path.exists(path):
            raise FileNotFoundError(f"{path} missing: run `make -C oracle`")
        lib = C.CDLL(path)
        self.lib = lib
        lib.or_half_to_float.argtypes = [C.c_uint16]; lib.or_half_to_float.restype = C.c_float
        lib.or_float_to_half.argtypes = [C.c_float]; lib.or_float_to_half.restype = C.c_uint16
        lib.or_half_to_float_vec.argtypes = [_u16p, C.c_size_t, _f32p]
        lib.or_float_to_half_vec.argtypes = [_f32p, C.c_size_t, _u16p]
        lib.or_gen_case.argtypes = [C.c_uint, C.c_int, C.c_int, C.c_int, _f32p, _f32p, _u16p]
        lib.or_selftest_seed.argtypes = [C.c_int] * 4; lib.or_selftest_seed.restype = C.c_uint
        lib.or_fill_fast.argtypes = [_f32p, C.c_size_t, C.c_uint64]
        lib.or_bench_query.argtypes = [C.c_int, C.c_int, _u16p]
        lib.or_quantize.argtypes = [_f32p, C.c_int, C.c_int, C.c_int, C.c_int, _u8p, _u16p]
        lib.or_dequant.argtypes = [_u8p, _u16p, C.c_int, C.c_int, C.c_int, C.c_int, _f32p]
        lib.or_round_to_half.argtypes = [_f32p, C.c_size_t, _f32p]
        for fn in ("or_quantize_kchan", "or_quantize_vtok"):
            getattr(lib, fn).argtypes = [_f32p, C.c_int, C.c_int, C.c_int, C.c_int, _u8p, _u16p]
        for fn in ("or_dequant_kchan", "or_dequant_vtok"):
            getattr(lib, fn).argtypes = [_u8p, _u16p, C.c_int, C.c_int, C.c_int, C.c_int, _f32p]
        lib.or_quantize_f8.argtypes = [_f32p, C.c_int, C.c_int, C.c_int, _u8p, _u16p]
        lib.or_dequant_f8.argtypes = [_u8p, _u16p, C.c_int, C.c_int, C.c_int, _f32p]
        lib.or_e4m3_encode_vec.argtypes = [_f32p, C.c_size_t, _u8p]
        lib.or_e4m3_decode_vec.argtypes = [_u8p, C.c_size_t, _f32p]
        lib.or_float_to_bf16_vec.argtypes = [_f32p, C.c_size_t, _u16p]
        lib.or_reference.argtypes = [_f32p, _f32p, _u16p, C.c_int, C.c_int, C.c_int, _f32p]
        lib.or_reference_mt.argtypes = [_f32p, _f32p, _u16p, C.c_int, C.c_int, C.c_int, _f32p, C.c_int]
        lib.or_combine.argtypes = [_f32p, C.c_int, C.c_int, C.c_int, _u16p]
        lib.or_partial.argtypes = [_f32p, _f32p, _u16p, C.c_int, C.c_int, C.c_int, C.c_int,
                                   C.c_int, C.c_int, _f32p]
        lib.or_reference_gqa.argtypes = [_f32p, _f32p, _u16p, _i32p, C.c_int, C.c_int, C.c_int,
                                         C.c_int, C.c_int, _f32p]

    # -- conversions
    def f2h(self, x: np.ndarray) -> np.ndarray:
        x = np.ascontiguousarray(x, np.float32).ravel()
        out = np.empty(x.size, np.uint16)
        self.lib.or_float_to_half_vec(x, x.size, out)
        return out

    def h2f(self, h: np.ndarray) -> np.ndarray:
        h = np.ascontiguousarray(h, np.uint16).ravel()
        out = np.empty(h.size, np.float32)
        self.lib.or_half_to_float_vec(h, h.size, out)
        return out

    # -- data
    def gen_case(self, seed: int, H: int, L: int, D: int):
        n = H * L * D
        kx = np.empty(n, np.float32); vx = np.empty(n, np.float32); q = np.empty(H * D, np.uint16)
        self.lib.or_gen_case(seed, H, L, D, kx, vx, q)
        return kx, vx, q

    def selftest_seed(self, H, L, D, S) -> int:
        return int(self.lib.or_selftest_seed(H, L, D, S))

    def fill_fast(self, n: int, seed: int) -> np.ndarray:
        v = np.empty(n, np.float32)
        self.lib.or_fill_fast(v, n, seed)
        return v

    def bench_query(self, H: int, D: int) -> np.ndarray:
        q = np.empty(H * D, np.uint16)
        self.lib.or_bench_query(H, D, q)
        return q

    # -- path
    def quantize(self, x: np.ndarray, H, L, D, bits):
        x = np.ascontiguousarray(x, np.float32).ravel()
        codes = np.zeros(payload_bytes(bits, H * L * D), np.uint8)
        scales = np.empty(H * L * (D // GROUP), np.uint16)
        self.lib.or_quantize(x, H, L, D, bits, codes, scales)
        return codes, scales

    def dequant(self, codes, scales, H, L, D, bits) -> np.ndarray:
        out = np.empty(H * L * D, np.float32)
        self.lib.or_dequant(np.ascontiguousarray(codes, np.uint8), np.ascontiguousarray(scales, np.uint16),
                            H, L, D, bits, out)
        return out

    def quantize_kchan(self, x: np.ndarray, H, L, D, bits):
        """q4c+ K: scales per (head, channel) over the head's L positions, [H][D]."""
        x = np.ascontiguousarray(x, np.float32).ravel()
        codes = np.zeros(payload_bytes(bits, H * L * D), np.uint8)
        scales = np.empty(H * D, np.uint16)
        self.lib.or_quantize_kchan(x, H, L, D, bits, codes, scales)
        return codes, scales

    def quantize_vtok(self, x: np.ndarray, H, L, D, bits):
        """q4c+ V: one scale per row, [H][L]."""
        x = np.ascontiguousarray(x, np.float32).ravel()
        codes = np.zeros(payload_bytes(bits, H * L * D), np.uint8)
        scales = np.empty(H * L, np.uint16)
        self.lib.or_quantize_vtok(x, H, L, D, bits, codes, scales)
        return codes, scales

    def dequant_kchan(self, codes, scales, H, L, D, bits) -> np.ndarray:
        out = np.empty(H * L * D, np.float32)
        self.lib.or_dequant_kchan(np.ascontiguousarray(codes, np.uint8), np.ascontiguousarray(scales, np.uint16),
                                  H, L, D, bits, out)
        return out

    def dequant_vtok(self, codes, scales, H, L, D, bits) -> np.ndarray:
        out = np.empty(H * L * D, np.float32)
        self.lib.or_dequant_vtok(np.ascontiguousarray(codes, np.uint8), np.ascontiguousarray(scales, np.uint16),
                                 H, L, D, bits, out)
        return out

    def quantize_f8(self, x: np.ndarray, H, L, D):
        x = np.ascontiguousarray(x, np.float32).ravel()
        codes = np.empty(H * L * D, np.uint8)
        scales = np.empty(H * L * (D // GROUP), np.uint16)
        self.lib.or_quantize_f8(x, H, L, D, codes, scales)
        return codes, scales

    def dequant_f8(self, codes, scales, H, L, D) -> np.ndarray:
        out = np.empty(H * L * D, np.float32)
        self.lib.or_dequant_f8(np.ascontiguousarray(codes, np.uint8), np.ascontiguousarray(scales, np.uint16),
                               H, L, D, out)
        return out

    def e4m3_encode(self, x) -> np.ndarray:
        x = np.ascontiguousarray(x, np.float32).ravel()
        out = np.empty(x.size, np.uint8)
        self.lib.or_e4m3_encode_vec(x, x.size, out)
        return out

    def e4m3_decode(self, c) -> np.ndarray:
        c = np.ascontiguousarray(c, np.uint8).ravel()
        out = np.empty(c.size, np.float32)
        self.lib.or_e4m3_decode_vec(c, c.size, out)
        return out

    def f2bf(self, x) -> np.ndarray:
        """bf16 bit patterns (round to nearest even)."""
        x = np.ascontiguousarray(x, np.float32).ravel()
        out = np.empty(x.size, np.uint16)
        self.lib.or_float_to_bf16_vec(x, x.size, out)
        return out

    def round_to_half(self, x) -> np.ndarray:
        x = np.ascontiguousarray(x, np.float32).ravel()
        out = np.empty_like(x)
        self.lib.or_round_to_half(x, x.size, out)
        return out

    def reference(self, kd, vd, q, H, L, D, threads: int = 1) -> np.ndarray:
        out = np.empty(H * D, np.float32)
        kd = np.ascontiguousarray(kd, np.float32); vd = np.ascontiguousarray(vd, np.float32)
        q = np.ascontiguousarray(q, np.uint16)
        if threads > 1:
            self.lib.or_reference_mt(kd, vd, q, H, L, D, out, threads)
        else:
            self.lib.or_reference(kd, vd, q, H, L, D, out)
        return out

    def combine(self, ws, H, S, D) -> np.ndarray:
        out = np.empty(H * D, np.uint16)
        self.lib.or_combine(np.ascontiguousarray(ws, np.float32), H, S, D, out)
        return out

    def partial(self, kd, vd, q, H, L, D, h, j0, j1) -> np.ndarray:
        slot = np.empty(D + 2, np.float32)
        self.lib.or_partial(np.ascontiguousarray(kd, np.float32), np.ascontiguousarray(vd, np.float32),
                            np.ascontiguousarray(q, np.uint16), H, L, D, h, j0, j1, slot)
        return slot

    def reference_gqa(self, kd, vd, q, lens, B, Hq, Hkv, Lmax, D) -> np.ndarray:
        out = np.empty(B * Hq * D, np.float32)
        self.lib.or_reference_gqa(np.ascontiguousarray(kd, np.float32), np.ascontiguousarray(vd, np.float32),
                                  np.ascontiguousarray(q, np.uint16), np.ascontiguousarray(lens, np.int32),
                                  B, Hq, Hkv, Lmax, D, out)
        return out

    # -- one selftest case's exact inputs (src/voltattn.cu:838-861)
    def case_inputs(self, fmt: str, H, L, D, seed):
        """Returns dict with the host data a case uploads and the exact values
        the reference attends over: kx/vx fp32, q fp16 bits, kd/vd fp32 and,
        for quantized formats, codes and scales of K and V."""
        kx, vx, q = self.gen_case(seed, H, L, D)
        d = {"kx": kx, "vx": vx, "q": q}
        if fmt.startswith("f16"):
            d["kd"] = self.round_to_half(kx); d["vd"] = self.round_to_half(vx)
        else:
            bits = BITS[fmt]
            kc, ks = self.quantize(kx, H, L, D, bits)
            vc, vs = self.quantize(vx, H, L, D, bits)
            d.update(kc=kc, ks=ks, vc=vc, vs=vs,
                     kd=self.dequant(kc, ks, H, L, D, bits), vd=self.dequant(vc, vs, H, L, D, bits))
        return d


class RefLib:
    """The reference's own host functions (and, on a GPU box, kernels)."""

    def __init__(self, path: str = REF_SO):
        if not os.path.exists(path):
            raise FileNotFoundError(f"{path} missing: built by `make -C oracle ref` where the reference source exists")
        lib = C.CDLL(path)
        self.lib = lib
        lib.ref_float2half.argtypes = [C.c_float]; lib.ref_float2half.restype = C.c_uint16
        lib.ref_half2float.argtypes = [C.c_uint16]; lib.ref_half2float.restype = C.c_float
        lib.ref_float2half_vec.argtypes = [_f32p, C.c_size_t, _u16p]
        lib.ref_half2float_vec.argtypes = [_u16p, C.c_size_t, _f32p]
        lib.ref_quantize.argtypes = [_f32p, C.c_int, C.c_int, C.c_int, C.c_int, _u8p, _u16p]
        lib.ref_dequant.argtypes = [_u8p, _u16p, C.c_int, C.c_int, C.c_int, C.c_int, _f32p]
        lib.ref_reference.argtypes = [_f32p, _f32p, _u16p, C.c_int, C.c_int, C.c_int, _f32p]
        lib.ref_reference_mt.argtypes = [_f32p, _f32p, _u16p, C.c_int, C.c_int, C.c_int, _f32p, C.c_int]
        lib.ref_fill_fast.argtypes = [_f32p, C.c_size_t, C.c_uint64]
        lib.ref_launch.argtypes = [C.c_int] + [C.c_void_p] * 7 + [C.c_int] * 5
        lib.ref_launch.restype = C.c_int
        lib.ref_time_launches.argtypes = [C.c_int] + [C.c_void_p] * 4 + [C.c_int] + [C.c_void_p] * 3 + \
            [C.c_int] * 5 + [C.POINTER(C.c_float)]
        lib.ref_time_launches.restype = C.c_int
        lib.ref_probe_ceiling.restype = C.c_double
        lib.ref_selftest.restype = C.c_int

    def quantize(self, x, H, L, D, bits):
        x = np.ascontiguousarray(x, np.float32).ravel()
        codes = np.zeros(payload_bytes(bits, H * L * D), np.uint8)
        scales = np.empty(H * L * (D // GROUP), np.uint16)
        self.lib.ref_quantize(x, H, L, D, bits, codes, scales)
        return codes, scales

    def dequant(self, codes, scales, H, L, D, bits):
        out = np.empty(H * L * D, np.float32)
        self.lib.ref_dequant(np.ascontiguousarray(codes, np.uint8), np.ascontiguousarray(scales, np.uint16),
                             H, L, D, bits, out)
        return out

    def reference(self, kd, vd, q, H, L, D, threads: int = 1):
        out = np.empty(H * D, np.float32)
        args = (np.ascontiguousarray(kd, np.float32), np.ascontiguousarray(vd, np.float32),
                np.ascontiguousarray(q, np.uint16), H, L, D, out)
        if threads > 1:
            self.lib.ref_reference_mt(*args, threads)
        else:
            self.lib.ref_reference(*args)
        return out

    def time_launches(self, fmt: int, caches, q_ptr, out_ptr, ws_ptr, H, L, D, S, n):
        """Average ms of n back-to-back reference launch() calls (GPU box only),
        rotating over caches = [(K, V, scK, scV) device pointers]."""
        k = len(caches)
        arr = lambda i: (C.c_void_p * k)(*[c[i] for c in caches])  # noqa: E731
        has_scales = caches[0][2] is not None
        ms = C.c_float(0.0)
        rc = self.lib.ref_time_launches(fmt, arr(0), arr(1), arr(2) if has_scales else None,
                                        arr(3) if has_scales else None, k, q_ptr, out_ptr, ws_ptr, H, L, D, S, n,
                                        C.byref(ms))
        if rc != 0:
            raise RuntimeError(f"ref_time_launches failed ({rc})")
        return ms.value

    def fill_fast(self, n, seed):
        v = np.empty(n, np.float32)
        self.lib.ref_fill_fast(v, n, seed)
        return v

    def f2h(self, x):
        x = np.ascontiguousarray(x, np.float32).ravel()
        out = np.empty(x.size, np.uint16)
        self.lib.ref_float2half_vec(x, x.size, out)
        return out

    def h2f(self, h):
        h = np.ascontiguousarray(h, np.uint16).ravel()
        out = np.empty(h.size, np.float32)
        self.lib.ref_half2float_vec(h, h.size, out)
        return out
