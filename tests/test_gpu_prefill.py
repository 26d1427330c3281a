"""Prefill (va_prefill): Lq new tokens of one sequence, causal over the cache
whose last Lq rows are theirs, on the tcgen05 tensor cores. Checked against the
oracle's GQA restatement of the reference's per-head math
(src/voltattn.cu:769-794) run once per token with the token's visible length
L - Lq + 1 + i. No reference counterpart (the reference decodes one token)."""
import numpy as np
import pytest

from oracle.oracle import BITS

pytestmark = pytest.mark.gpu

# K and V are rounded to fp16 tile by tile (code * scale) and P is fp16 in the
# tensor-core product: the same bar as the decode kernels
ATOL, RTOL = 2e-3, 1e-3


@pytest.fixture(scope="module")
def va():
    import torch
    assert torch.cuda.is_available()
    import voltattn_b200
    return voltattn_b200


CASES = [  # fmt, Hq, Hkv, L, Lq
    ("q4+", 8, 2, 700, 300),   # 4 query heads per KV head, tokens not a multiple of 128
    ("q8+", 4, 4, 256, 256),   # the whole cache is new
    ("f16+", 2, 1, 1000, 130),
    ("q3+", 4, 2, 500, 129),
    ("q4", 4, 4, 128, 1),      # one token: a decode
    ("f16", 2, 2, 333, 77),
    ("q8", 2, 1, 1500, 200),
    ("q4+", 2, 2, 2049, 640),  # several token blocks, cache blocks past the diagonal
    ("bf16+", 4, 2, 600, 200),
    ("f8+", 4, 1, 777, 300),
    ("q4c+", 8, 2, 900, 260),  # per-channel K scales, per-row V scales
]


def cache_for(oracle, fmt, kx, vx, rows, D, L):
    """Device-side codes and scales plus the exact values the reference attends over."""
    if fmt.startswith("f16"):
        kb, vb = oracle.f2h(kx), oracle.f2h(vx)
        return kb, vb, None, None, oracle.round_to_half(kx), oracle.round_to_half(vx)
    if fmt == "bf16+":
        kb, vb = oracle.f2bf(kx), oracle.f2bf(vx)
        val = lambda b: (b.astype(np.uint32) << 16).view(np.float32)
        return kb, vb, None, None, val(kb), val(vb)
    if fmt == "q4c+":  # K scales per (KV head, channel), V scales per row
        H = rows // L
        kc, ks = oracle.quantize_kchan(kx, H, L, D, 4)
        vc, vs = oracle.quantize_vtok(vx, H, L, D, 4)
        return kc, vc, ks, vs, oracle.dequant_kchan(kc, ks, H, L, D, 4), oracle.dequant_vtok(vc, vs, H, L, D, 4)
    if fmt == "f8+":
        kc, ks = oracle.quantize_f8(kx, 1, rows, D)
        vc, vs = oracle.quantize_f8(vx, 1, rows, D)
        return kc, vc, ks, vs, oracle.dequant_f8(kc, ks, 1, rows, D), oracle.dequant_f8(vc, vs, 1, rows, D)
    bits = BITS[fmt]
    kc, ks = oracle.quantize(kx, 1, rows, D, bits)
    vc, vs = oracle.quantize(vx, 1, rows, D, bits)
    return kc, vc, ks, vs, oracle.dequant(kc, ks, 1, rows, D, bits), oracle.dequant(vc, vs, 1, rows, D, bits)


@pytest.mark.parametrize("staged", [True, False], ids=["staged", "unstaged"])
@pytest.mark.parametrize("case", CASES, ids=lambda c: "{}_Hq{}_Hkv{}_L{}_Lq{}".format(*c))
def test_prefill(va, oracle, case, staged):
    import torch
    fmt, Hq, Hkv, L, Lq = case
    D = 128
    rng = np.random.default_rng(Hq * 131 + Hkv * 17 + L + Lq)
    rows = Hkv * L
    kx, vx, _ = oracle.gen_case(int(rng.integers(1 << 30)), 1, rows, D)
    kc, vc, ks, vs, kd, vd = cache_for(oracle, fmt, kx, vx, rows, D, L)
    q = oracle.f2h(rng.standard_normal(Hq * Lq * D).astype(np.float32)).reshape(Hq, Lq, D)
    ref = np.empty((Hq, Lq, D), np.float32)
    for i in range(Lq):
        li = np.array([L - Lq + 1 + i], np.int32)
        ref[:, i] = oracle.reference_gqa(kd, vd, np.ascontiguousarray(q[:, i]).ravel(), li, 1, Hq, Hkv, L,
                                         D).reshape(Hq, D)
    dev = "cuda"
    as_dev = lambda a: torch.from_numpy(np.ascontiguousarray(a)).to(dev)
    K, V = as_dev(kc), as_dev(vc)
    sK = None if ks is None else as_dev(ks).view(torch.float16)
    sV = None if vs is None else as_dev(vs).view(torch.float16)
    qd = as_dev(q.ravel()).view(torch.float16)
    out = torch.full((Hq * Lq * D,), float("nan"), dtype=torch.float16, device=dev)
    b = va.DeviceBufs(K, V, sK, sV, qd, out)
    for _ in range(2):
        va.prefill(fmt, b, Hq, Hkv, L, Lq, D, staged=staged)
        torch.cuda.synchronize()
        got = out.float().cpu().numpy().reshape(Hq, Lq, D)
        err = np.abs(got - ref)
        bad = ~(err <= ATOL + RTOL * np.abs(ref))
        assert not bad.any(), f"{case}: {bad.sum()} bad, maxerr {np.nanmax(err):.3e}"
    assert va.device_error() == 0


def test_prefill_rejects_unsupported(va):
    import torch
    Hq, Hkv, L, Lq = 2, 2, 64, 8
    K = torch.zeros(Hkv * L * 64, dtype=torch.uint8, device="cuda")
    s = torch.zeros(Hkv * L * 2, dtype=torch.float16, device="cuda")
    q = torch.zeros(Hq * Lq * 64, dtype=torch.float16, device="cuda")
    b = va.DeviceBufs(K, K, s, s, q, q.clone())
    with pytest.raises(RuntimeError):  # D = 64
        va.prefill("q4+", b, Hq, Hkv, L, Lq, 64)
    with pytest.raises(RuntimeError):  # more new tokens than cache rows
        va.prefill("q4+", b, Hq, Hkv, 4, Lq, 128)


PAGED = [  # fmt, Hq, Hkv, L, Lq, page_rows
    ("q4+", 8, 2, 700, 300, 64),
    ("q8+", 4, 4, 1000, 129, 48),   # pages not a multiple of the 128-row block
    ("f16+", 2, 1, 513, 513, 256),
    ("q3+", 4, 2, 400, 77, 32),
]


@pytest.mark.parametrize("staged", [True, False], ids=["staged", "unstaged"])
@pytest.mark.parametrize("case", PAGED, ids=lambda c: "{}_Hq{}_Hkv{}_L{}_Lq{}_P{}".format(*c))
def test_prefill_paged(va, oracle, case, staged):
    """The contiguous case's cache scattered into a shuffled page pool whose
    unused pages carry nan scales (or nan fp16 rows): the output must match
    the oracle exactly as for the contiguous layout."""
    import torch
    fmt, Hq, Hkv, L, Lq, P = case
    D = 128
    rng = np.random.default_rng(Hq * 7 + L + P)
    rows = Hkv * L
    kx, vx, _ = oracle.gen_case(int(rng.integers(1 << 30)), 1, rows, D)
    kc, vc, ks, vs, kd, vd = cache_for(oracle, fmt, kx, vx, rows, D, L)
    q = oracle.f2h(rng.standard_normal(Hq * Lq * D).astype(np.float32)).reshape(Hq, Lq, D)
    ref = np.empty((Hq, Lq, D), np.float32)
    for i in range(Lq):
        ref[:, i] = oracle.reference_gqa(kd, vd, np.ascontiguousarray(q[:, i]).ravel(),
                                         np.array([L - Lq + 1 + i], np.int32), 1, Hq, Hkv, L, D).reshape(Hq, D)
    max_pages = (L + P - 1) // P
    num_pages = max_pages + 3
    table = rng.permutation(num_pages)[:max_pages].astype(np.int32)

    def scatter(arr, per_row, fill):
        a = arr.reshape(Hkv, L, per_row)
        pool = np.full((num_pages, Hkv, P, per_row), fill, arr.dtype)
        for j in range(max_pages):
            r1 = min((j + 1) * P, L)
            pool[table[j], :, :r1 - j * P] = a[:, j * P:r1]
        return pool.reshape(-1)

    nan16 = np.uint16(0x7E00)
    if fmt.startswith("f16"):
        K, V = scatter(kc.view(np.uint16), D, nan16), scatter(vc.view(np.uint16), D, nan16)
        sK = sV = None
    else:
        rb = kc.size // rows
        K, V = scatter(kc, rb, 0), scatter(vc, rb, 0)
        sK, sV = scatter(ks.view(np.uint16), 2, nan16), scatter(vs.view(np.uint16), 2, nan16)
    as_dev = lambda a: torch.from_numpy(np.ascontiguousarray(a)).cuda()
    Kd, Vd = as_dev(K), as_dev(V)
    sKd = None if sK is None else as_dev(sK).view(torch.float16)
    sVd = None if sV is None else as_dev(sV).view(torch.float16)
    qd = as_dev(q.ravel()).view(torch.float16)
    out = torch.full((Hq * Lq * D,), float("nan"), dtype=torch.float16, device="cuda")
    va.prefill_paged(fmt, va.DeviceBufs(Kd, Vd, sKd, sVd, qd, out), as_dev(table), max_pages, P, num_pages, Hq, Hkv,
                     L, Lq, D, staged=staged)
    torch.cuda.synchronize()
    got = out.float().cpu().numpy().reshape(Hq, Lq, D)
    err = np.abs(got - ref)
    bad = ~(err <= ATOL + RTOL * np.abs(ref))
    assert not bad.any(), f"{case}: {bad.sum()} bad, maxerr {np.nanmax(err):.3e}"
    assert va.device_error() == 0
