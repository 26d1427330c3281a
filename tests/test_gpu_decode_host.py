"""va_decode_host: a decode step with the query and the output in pinned host
memory, captured once per argument set into a CUDA graph. Its output must equal
va_decode's (the same kernels on the same data) on every call, including calls
that replay the graph with new query values, and on the legacy default stream."""
import numpy as np
import pytest

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module")
def va():
    import torch
    assert torch.cuda.is_available()
    import voltattn_b200
    return voltattn_b200


@pytest.mark.parametrize("fmt", ["q4+", "q8+", "f16+", "q3+"])
@pytest.mark.parametrize("on_stream", [True, False])
def test_decode_host_matches_decode(va, oracle, fmt, on_stream):
    import torch
    H, L, D = 8, 3000, 128
    S = va.suggest_splits(fmt, H, L, D)
    kx, vx, _ = oracle.gen_case(L + H, H, L, D)
    bits = 16 if fmt.startswith("f16") else va.qbits(fmt)
    if bits == 16:
        K, V, sK, sV = torch.from_numpy(kx).cuda().half(), torch.from_numpy(vx).cuda().half(), None, None
    else:
        K, sK = va.quantize(torch.from_numpy(kx).cuda(), bits, H, L, D)
        V, sV = va.quantize(torch.from_numpy(vx).cuda(), bits, H, L, D)
    q_dev = torch.empty(H * D, dtype=torch.float16, device="cuda")
    out_dev = torch.empty_like(q_dev)
    b = va.DeviceBufs(K, V, sK, sV, q_dev, out_dev, va.new_workspace(H, D, S))
    q_pin = torch.empty(H * D, dtype=torch.float16).pin_memory()
    out_pin = torch.empty(H * D, dtype=torch.float16).pin_memory()
    stream = torch.cuda.Stream() if on_stream else None
    rng = np.random.default_rng(3)
    for step in range(3):  # first call captures; later calls replay with new q
        qv = torch.from_numpy(rng.standard_normal(H * D).astype(np.float32)).half()
        q_pin.copy_(qv)
        out_pin.fill_(float("nan"))
        if step < 2:
            va.decode_host(fmt, b, q_pin, out_pin, H, L, D, S, stream)
        else:  # the bound form replays the same cached graph
            va.HostStep(fmt, b, q_pin, out_pin, H, L, D, S, stream)()
        got = out_pin.clone()
        want = va.decode(fmt, K, V, sK, sV, qv.cuda(), H, L, D, S).cpu()
        assert torch.equal(got, want), f"{fmt} step {step}: differs from va_decode"
    assert va.device_error() == 0


def test_pageable_host_memory_is_rejected_before_any_launch(va):
    """Ordinary (pageable) host memory cannot be reached by a kernel: the host
    entry points refuse it with VA_ERR_INVALID instead of launching on it."""
    import ctypes as C

    import torch
    lib = va.lib()
    H, L, D, S = 2, 64, 128, 1
    K, sK = va.quantize(torch.randn(H * L * D, device="cuda"), 8, H, L, D)
    q_dev = torch.empty(H * D, dtype=torch.float16, device="cuda")
    out_dev = torch.empty_like(q_dev)
    b = va.DeviceBufs(K, K, sK, sK, q_dev, out_dev, va.new_workspace(H, D, S))
    pageable = np.zeros(H * D + 64, dtype=np.float16)
    off = (-pageable.ctypes.data) % 16 // 2  # a 16-byte aligned view, so only pinning is wrong
    host = pageable[off:off + H * D]
    pinned = torch.empty(H * D, dtype=torch.float16).pin_memory()
    bb = b.va()
    ws = b.ws
    fmt = int(va.Fmt.parse("q8+"))
    for q_ptr, out_ptr in ((host.ctypes.data, pinned.data_ptr()), (pinned.data_ptr(), host.ctypes.data)):
        rc = lib.va_decode_host(fmt, C.byref(bb), q_ptr, out_ptr, H, L, D, S, ws.data_ptr(), ws.numel() * ws.element_size(), None)
        assert rc == 1, rc  # VA_ERR_INVALID
    assert lib.va_copy_small(q_dev.data_ptr(), host.ctypes.data, H * D * 2, None) == 1
    assert lib.va_copy_small(host.ctypes.data, q_dev.data_ptr(), H * D * 2, None) == 1
    torch.cuda.synchronize()
    assert va.device_error() == 0
