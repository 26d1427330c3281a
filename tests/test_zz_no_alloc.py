"""va_decode_noalloc: the decode entry point for callers that cannot allocate
device memory (hosts that own the whole memory pool or forbid allocation
after start-up). It keeps its workspace in a fixed array inside the library.
This test calls it through the C ABI and checks it against va_decode, the
entry point with a caller-provided workspace, on two calls in a row (the
second call reuses the array with the first call's leftovers in it). It runs
last (file name) and needs nothing from the other tests."""
import ctypes as C

import pytest

pytestmark = pytest.mark.gpu

ATOL, RTOL = 2e-3, 1e-3  # the tolerance of the other decode tests


def test_noalloc_matches_decode_two_calls():
    import torch
    assert torch.cuda.is_available()
    import voltattn_b200 as va
    lib = va.lib()
    torch.manual_seed(7)
    H, L, D, S = 8, 1031, 128, 5
    dev = torch.device("cuda", 0)
    for fmt, bits in (("q8+", 8), ("q4+", 4), ("f16+", 16)):
        kx = torch.randn(H * L * D, device=dev)
        vx = torch.randn(H * L * D, device=dev)
        if bits == 16:
            K, V, sK, sV = kx.half(), vx.half(), None, None
        else:
            K, sK = va.quantize(kx, bits, H, L, D)
            V, sV = va.quantize(vx, bits, H, L, D)
        for call in range(2):
            q = torch.randn(H * D, device=dev).half()
            want = torch.empty(H * D, dtype=torch.float16, device=dev)
            va.launch(fmt, va.DeviceBufs(K, V, sK, sV, q, want, va.new_workspace(H, D, S, dev)), H, L, D, S)
            got = torch.full((H * D,), float("nan"), dtype=torch.float16, device=dev)
            b = va.DeviceBufs(K, V, sK, sV, q, got).va()
            stream = torch.cuda.current_stream().cuda_stream
            assert lib.va_decode_noalloc(int(va.Fmt.parse(fmt)), C.byref(b), H, L, D, S, stream) == 0
            torch.cuda.synchronize()
            err = (got.float() - want.float()).abs()
            assert bool((err <= ATOL + RTOL * want.float().abs()).all()), (fmt, call, float(err.max()))
    assert va.device_error() == 0


def test_noalloc_rejects_sizes_beyond_its_array():
    import torch
    import voltattn_b200 as va
    lib = va.lib()
    H, L, D, S = 32, 70000, 128, 4096  # needs far more than the 4 MiB array
    t = torch.empty(16, dtype=torch.uint8, device="cuda")
    b = va.VaBufs(t.data_ptr(), t.data_ptr(), t.data_ptr(), t.data_ptr(), t.data_ptr(), t.data_ptr())
    assert lib.va_decode_noalloc(int(va.Fmt.Q8M), C.byref(b), H, L, D, S, None) == 7  # VA_ERR_TOO_LARGE
