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


def _cache(va, torch, fmt, H, L, D, dev):
    kx = torch.randn(H * L * D, device=dev)
    vx = torch.randn(H * L * D, device=dev)
    if fmt == "f16+":
        return kx.half(), vx.half(), None, None
    if fmt == "q4c+":  # per-channel K scales, per-row V scales
        K, sK = va.quantize_kchan(kx, 4, H, L, D)
        V, sV = va.quantize_vtok(vx, 4, H, L, D)
        return K, V, sK, sV
    bits = {"q8+": 8, "q4+": 4, "q3+": 3}[fmt]
    K, sK = va.quantize(kx, bits, H, L, D)
    V, sV = va.quantize(vx, bits, H, L, D)
    return K, V, sK, sV


@pytest.mark.parametrize("fmt", ["q8+", "q4+", "q3+", "q4c+", "f16+"])
def test_noalloc_matches_decode_two_calls(fmt):
    import torch
    assert torch.cuda.is_available()
    import voltattn_b200 as va
    lib = va.lib()
    torch.manual_seed(7)
    H, L, D = 8, 1031, 128
    dev = torch.device("cuda", 0)
    K, V, sK, sV = _cache(va, torch, fmt, H, L, D, dev)
    # The second call uses fewer splits, so its counters sit inside the first
    # call's slot floats: it is right only if the entry point clears them.
    for call, S in enumerate((5, 2)):
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
