"""Batched grouped-query decode (va_decode_gqa) against the oracle's GQA
restatement (or_reference_gqa: query head hq of sequence b attends over KV
head hq / (Hq/Hkv) of that sequence, positions [0, lens[b])). Rows past
lens[b] hold nan scales / nan fp16 values and must never leak into a result.
No reference counterpart: the reference is batch 1, one KV head per head."""
import numpy as np
import pytest

from oracle.oracle import BITS

pytestmark = pytest.mark.gpu

ATOL, RTOL = 2e-3, 1e-3


@pytest.fixture(scope="module")
def va():
    import torch
    assert torch.cuda.is_available()
    import voltattn_b200
    return voltattn_b200


CASES = [  # B, Hq, Hkv, Lmax, D, S
    (3, 8, 2, 700, 128, 3),
    (2, 8, 8, 257, 64, 2),
    (4, 16, 2, 1031, 128, 4),
    (2, 16, 2, 513, 64, 1),
    (5, 4, 1, 96, 128, 7),
    (3, 8, 4, 600, 128, 2),   # 2 query heads per KV head
]


@pytest.mark.parametrize("fmt", ["f16+", "q8+", "q4+", "q3+"])
@pytest.mark.parametrize("case", CASES, ids=lambda c: "B{}_Hq{}_Hkv{}_L{}_D{}_S{}".format(*c))
def test_gqa(va, oracle, fmt, case):
    import torch
    B, Hq, Hkv, Lmax, D, S = case
    rng = np.random.default_rng(B * 1000 + Hq * 10 + Lmax)
    lens = rng.integers(1, Lmax + 1, size=B).astype(np.int32)
    lens[0] = Lmax
    rows = B * Hkv * Lmax
    kx, vx, _ = oracle.gen_case(int(rng.integers(1 << 30)), 1, rows, D)
    q = oracle.f2h(rng.standard_normal(B * Hq * D).astype(np.float32))
    valid = np.zeros((B, Hkv, Lmax), bool)
    for b in range(B):
        valid[b, :, :lens[b]] = True
    valid = valid.reshape(-1)
    if fmt == "f16+":
        kd, vd = oracle.round_to_half(kx), oracle.round_to_half(vx)
        K = torch.from_numpy(kx).cuda().half().view(rows, D)
        V = torch.from_numpy(vx).cuda().half().view(rows, D)
        K[torch.from_numpy(~valid).cuda()] = float("nan")
        V[torch.from_numpy(~valid).cuda()] = float("nan")
        sK = sV = None
    else:
        bits = BITS[fmt]
        kc, ks = oracle.quantize(kx, 1, rows, D, bits)
        vc, vs = oracle.quantize(vx, 1, rows, D, bits)
        kd, vd = oracle.dequant(kc, ks, 1, rows, D, bits), oracle.dequant(vc, vs, 1, rows, D, bits)
        K, V = torch.from_numpy(kc).cuda(), torch.from_numpy(vc).cuda()
        sK = torch.from_numpy(ks).cuda().view(torch.float16).view(rows, -1)
        sV = torch.from_numpy(vs).cuda().view(torch.float16).view(rows, -1)
        sK[torch.from_numpy(~valid).cuda()] = float("nan")
        sV[torch.from_numpy(~valid).cuda()] = float("inf")
    ref = oracle.reference_gqa(kd, vd, q, lens, B, Hq, Hkv, Lmax, D)
    out = torch.full((B * Hq * D,), float("nan"), dtype=torch.float16, device="cuda")
    ws = torch.zeros(va.gqa_workspace_bytes(B, Hq, D, S), dtype=torch.uint8, device="cuda")
    qd = torch.from_numpy(q).cuda().view(torch.float16)
    lens_d = torch.from_numpy(lens).cuda()
    for _ in range(2):  # second call reuses the workspace (counters left at zero)
        va.decode_gqa(fmt, va.DeviceBufs(K, V, sK, sV, qd, out, ws), lens_d, B, Hq, Hkv, Lmax, D, S)
        torch.cuda.synchronize()
        got = out.float().cpu().numpy()
        err = np.abs(got - ref)
        bad = ~(err <= ATOL + RTOL * np.abs(ref))
        assert not bad.any(), f"{fmt} {case}: {bad.sum()} bad, maxerr {np.nanmax(err):.3e}"
    assert va.device_error() == 0


def test_gqa_rejects_bad_group(va):
    import ctypes as C
    import torch
    t = torch.empty(64, dtype=torch.uint8, device="cuda")
    p = t.data_ptr()
    b = va.VaBufs(p, p, p, p, p, p)
    lib = va.lib()
    assert lib.va_decode_gqa(5, C.byref(b), p, 1, 12, 4, 64, 128, 1, p, 1 << 20, None) == 5  # G = 3
    assert lib.va_decode_gqa(5, C.byref(b), p, 1, 10, 4, 64, 128, 1, p, 1 << 20, None) == 1  # Hq % Hkv
    assert lib.va_decode_gqa(4, C.byref(b), p, 1, 8, 4, 64, 128, 1, p, 1 << 20, None) == 5   # plain q4
