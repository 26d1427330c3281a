"""KV append (va_append_kv): appending rows one position at a time writes the
same bytes as quantizing the whole cache at once (the reference's quantize(),
src/voltattn.cu:705-745, is row-local), and an append + grouped-query decode
loop matches the oracle."""
import numpy as np
import pytest

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module")
def va():
    import torch
    assert torch.cuda.is_available()
    import voltattn_b200
    return voltattn_b200


@pytest.mark.parametrize("bits", [8, 4, 3, 16])
@pytest.mark.parametrize("D", [128, 64])
def test_append_equals_whole_quantize(va, bits, D):
    import torch
    B, Hkv, Lcap = 3, 2, 24
    rows = B * Hkv * Lcap
    g = torch.Generator(device="cuda").manual_seed(bits * 100 + D)
    x = torch.randn(B, Hkv, Lcap, D, generator=g, device="cuda")
    x[0, 1, 5, :64] *= 1e-7  # an underflowing fp16 scale
    if bits == 16:
        want = x.half().reshape(-1).view(torch.uint8)
        codes = torch.zeros(rows * D * 2, dtype=torch.uint8, device="cuda")
        scales = None
    else:
        want, want_s = va.quantize(x.reshape(-1).contiguous(), bits, 1, rows, D)
        codes = torch.zeros_like(want)
        scales = torch.zeros(rows * (D // 64), dtype=torch.float16, device="cuda")
    # sequence b starts at length b and grows; positions >= Lcap are skipped
    pos = torch.arange(B, dtype=torch.int32, device="cuda")
    for step in range(Lcap + 2):
        p = pos.clone()
        new = torch.stack([x[b, :, min(int(p[b]), Lcap - 1)] for b in range(B)]).contiguous()
        va.append_kv(new, bits, codes, scales, B, Hkv, Lcap, D, p)
        pos += 1
    # rows below each sequence's start were never appended: fill them directly
    for b in range(B):
        for t in range(b):
            r = torch.zeros(B, dtype=torch.int32, device="cuda") - 1
            r[b] = t
            new = x[:, :, t].contiguous()
            va.append_kv(new, bits, codes, scales, B, Hkv, Lcap, D, r)
    torch.cuda.synchronize()
    assert torch.equal(codes, want)
    if scales is not None:
        assert torch.equal(scales.view(torch.uint16), want_s.view(torch.uint16))


def test_append_then_decode_loop(va, oracle):
    import torch
    from oracle.oracle import BITS
    fmt, bits = "q4+", BITS["q4+"]
    B, Hq, Hkv, Lcap, D, S = 2, 8, 2, 300, 128, 3
    rng = np.random.default_rng(11)
    lens = np.array([100, 37], np.int32)
    rows = B * Hkv * Lcap
    kx, vx, _ = oracle.gen_case(99, 1, rows, D)
    K = torch.zeros(rows * D // 2, dtype=torch.uint8, device="cuda")
    V = torch.zeros_like(K)
    sK = torch.zeros(rows * 2, dtype=torch.float16, device="cuda")
    sV = torch.zeros_like(sK)
    kt = torch.from_numpy(kx).cuda().view(B, Hkv, Lcap, D)
    vt = torch.from_numpy(vx).cuda().view(B, Hkv, Lcap, D)
    for t in range(int(lens.max())):  # prefill positions below each length
        p = torch.tensor([t if t < lens[b] else -1 for b in range(B)], dtype=torch.int32, device="cuda")
        va.append_kv(kt[:, :, t].contiguous(), bits, K, sK, B, Hkv, Lcap, D, p)
        va.append_kv(vt[:, :, t].contiguous(), bits, V, sV, B, Hkv, Lcap, D, p)
    ws = torch.zeros(va.gqa_workspace_bytes(B, Hq, D, S), dtype=torch.uint8, device="cuda")
    out = torch.empty(B * Hq * D, dtype=torch.float16, device="cuda")
    for step in range(3):  # decode loop: append the new token, then attend
        p = torch.from_numpy(lens).cuda()
        va.append_kv(torch.stack([kt[b, :, lens[b]] for b in range(B)]).contiguous(), bits, K, sK, B, Hkv, Lcap, D, p)
        va.append_kv(torch.stack([vt[b, :, lens[b]] for b in range(B)]).contiguous(), bits, V, sV, B, Hkv, Lcap, D, p)
        lens = lens + 1
        q = oracle.f2h(rng.standard_normal(B * Hq * D).astype(np.float32))
        va.decode_gqa(fmt, va.DeviceBufs(K, V, sK, sV, torch.from_numpy(q).cuda().view(torch.float16), out, ws),
                      torch.from_numpy(lens).cuda(), B, Hq, Hkv, Lcap, D, S)
        torch.cuda.synchronize()
        kc, ks = oracle.quantize(kx, 1, rows, D, bits)
        vc, vs = oracle.quantize(vx, 1, rows, D, bits)
        ref = oracle.reference_gqa(oracle.dequant(kc, ks, 1, rows, D, bits), oracle.dequant(vc, vs, 1, rows, D, bits),
                                   q, lens, B, Hq, Hkv, Lcap, D)
        got = out.float().cpu().numpy()
        err = np.abs(got - ref)
        assert (err <= 2e-3 + 1e-3 * np.abs(ref)).all(), (step, float(err.max()))


def test_copy_small_pinned_and_device(va):
    """va_copy_small between device memory and device-mapped pinned host memory."""
    import torch
    src = torch.randn(4096).half().pin_memory()
    dev = torch.empty(4096, dtype=torch.float16, device="cuda")
    back = torch.empty(4096, dtype=torch.float16).pin_memory()
    va.copy_small(dev, src)
    va.copy_small(back, dev)
    torch.cuda.synchronize()
    assert torch.equal(back, src)
    d2 = torch.empty_like(dev)
    va.copy_small(d2, dev)
    torch.cuda.synchronize()
    assert torch.equal(d2, dev)
