"""Failure detection of the split-L exchange on one GPU, without a GPU fault:
the peer waits are bounded, and a wait made to run out (a second rank's
buffer that nothing ever publishes to) must end the kernel with the
peer-wait device error, leave the output untouched, and return within a few
seconds. Only one kernel runs; nothing waits on another kernel. Also the
one-launch split-L entry point with a single rank, against va_decode."""
import ctypes as C
import time

import pytest

pytestmark = pytest.mark.gpu

K_ERR_PEER_WAIT = 4


@pytest.fixture(scope="module")
def va():
    import torch
    assert torch.cuda.is_available()
    import voltattn_b200
    return voltattn_b200


@pytest.fixture
def short_wait(va):
    va.set_peer_wait_limit(0.01)
    yield
    va.set_peer_wait_limit(1.0)


def _cache(va, H, L, D, seed=3):
    import torch
    g = torch.Generator(device="cuda").manual_seed(seed)
    K, sK = va.quantize(torch.randn(H * L * D, device="cuda", generator=g), 4, H, L, D)
    V, sV = va.quantize(torch.randn(H * L * D, device="cuda", generator=g), 4, H, L, D)
    q = torch.randn(H * D, device="cuda", generator=g).half()
    return K, V, sK, sV, q


def _buffers(va, R, H, D):
    import torch
    return [torch.zeros(va.exchange_buffer_bytes(R, H, D), dtype=torch.uint8, device="cuda") for _ in range(R)]


def test_exchange_wait_runs_out(va, short_wait):
    import torch
    H, D, R = 4, 128, 2
    bufs = _buffers(va, R, H, D)
    partial = torch.randn(H, D + 2, device="cuda")
    partial[:, 0] = 0.0
    partial[:, 1] = 1.0
    out = torch.full((H * D,), 7.0, dtype=torch.float16, device="cuda")
    t = time.time()
    va.exchange_combine(partial, H, D, R, 0, [b.data_ptr() for b in bufs], 1, out)
    torch.cuda.synchronize()
    assert time.time() - t < 5.0
    assert va.device_error() == K_ERR_PEER_WAIT
    assert bool((out == 7.0).all()), "a head whose peers never arrived must stay untouched"


def test_fused_splitl_wait_runs_out(va, short_wait):
    import torch
    H, L, D, R = 4, 1000, 128, 2
    K, V, sK, sV, q = _cache(va, H, L, D)
    bufs = _buffers(va, R, H, D)
    out = torch.full((H * D,), 7.0, dtype=torch.float16, device="cuda")
    S = 3
    b = va.DeviceBufs(K, V, sK, sV, q, out, va.new_workspace(H, D, S))
    arr = (C.c_void_p * R)(*[x.data_ptr() for x in bufs])
    t = time.time()
    va.decode_splitl("q4+", b, H, L, D, S, R, 0, arr, 1)
    torch.cuda.synchronize()
    assert time.time() - t < 5.0
    assert va.device_error() == K_ERR_PEER_WAIT
    assert bool((out == 7.0).all())


@pytest.mark.parametrize("fmt", ["q4+", "q8+", "q3+"])
def test_fused_splitl_single_rank_matches_decode(va, fmt):
    import torch
    H, L, D, S = 8, 3001, 128, 4
    g = torch.Generator(device="cuda").manual_seed(11)
    bits = va.qbits(fmt)
    K, sK = va.quantize(torch.randn(H * L * D, device="cuda", generator=g), bits, H, L, D)
    V, sV = va.quantize(torch.randn(H * L * D, device="cuda", generator=g), bits, H, L, D)
    bufs = _buffers(va, 1, H, D)
    arr = (C.c_void_p * 1)(bufs[0].data_ptr())
    # host-counted steps: both parity halves, then the first again; then a
    # fresh buffer with device-counted steps (epoch 0)
    fresh = _buffers(va, 1, H, D)
    arr0 = (C.c_void_p * 1)(fresh[0].data_ptr())
    for epoch, a in ((1, arr), (2, arr), (3, arr), (0, arr0), (0, arr0), (0, arr0)):
        q = torch.randn(H * D, device="cuda", generator=g).half()
        want = va.decode(fmt, K, V, sK, sV, q, H, L, D, S).float()
        out = torch.full((H * D,), float("nan"), dtype=torch.float16, device="cuda")
        va.decode_splitl(fmt, va.DeviceBufs(K, V, sK, sV, q, out, va.new_workspace(H, D, S)), H, L, D, S, 1, 0, a,
                         epoch)
        err = (out.float() - want).abs()
        assert bool((err <= 2e-3 + 1e-3 * want.abs()).all()), (fmt, epoch, float(err.max()))
