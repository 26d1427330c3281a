"""Multi-query decode (va_decode_multiquery): Q new tokens per sequence, causal
among themselves, against the oracle's GQA restatement run once per token with
the token's visible length lens[b] - (Q-1-i). Rows past lens[b] carry nan/inf
scales and must never leak. No reference counterpart (the reference decodes one
token per head)."""
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


CASES = [  # B, Hq, Hkv, Q, Lmax, S
    (3, 4, 4, 4, 500, 2),    # one query head per KV head, 4 tokens
    (2, 8, 4, 2, 700, 3),    # 2 heads x 2 tokens
    (2, 8, 2, 2, 600, 2),    # 4 heads x 2 tokens
    (2, 4, 4, 8, 300, 1),    # 8 tokens
    (3, 4, 4, 2, 1000, 4),   # 2 tokens
    (1, 32, 8, 2, 5000, 4),  # 4 x 2 at a longer length
]


@pytest.mark.parametrize("case", CASES, ids=lambda c: "B{}_Hq{}_Hkv{}_Q{}_L{}_S{}".format(*c))
def test_multiquery(va, oracle, case):
    import torch
    B, Hq, Hkv, Q, Lmax, S = case
    D, fmt = 128, "q4+"
    bits = BITS[fmt]
    rng = np.random.default_rng(B * 97 + Hq * 13 + Q * 7 + Lmax)
    lens = rng.integers(Q, Lmax + 1, size=B).astype(np.int32)
    lens[0] = Lmax
    rows = B * Hkv * Lmax
    kx, vx, _ = oracle.gen_case(int(rng.integers(1 << 30)), 1, rows, D)
    q = oracle.f2h(rng.standard_normal(B * Hq * Q * D).astype(np.float32)).reshape(B, Hq, Q, D)
    kc, ks = oracle.quantize(kx, 1, rows, D, bits)
    vc, vs = oracle.quantize(vx, 1, rows, D, bits)
    kd, vd = oracle.dequant(kc, ks, 1, rows, D, bits), oracle.dequant(vc, vs, 1, rows, D, bits)
    ref = np.empty((B, Hq, Q, D), np.float32)
    for i in range(Q):
        li = (lens - (Q - 1 - i)).astype(np.int32)
        ref[:, :, i] = oracle.reference_gqa(kd, vd, np.ascontiguousarray(q[:, :, i]).ravel(), li, B, Hq, Hkv,
                                            Lmax, D).reshape(B, Hq, D)
    valid = np.zeros((B, Hkv, Lmax), bool)
    for b in range(B):
        valid[b, :, :lens[b]] = True
    valid = torch.from_numpy(~valid.reshape(-1)).cuda()
    K, V = torch.from_numpy(kc).cuda(), torch.from_numpy(vc).cuda()
    sK = torch.from_numpy(ks).cuda().view(torch.float16).view(rows, -1)
    sV = torch.from_numpy(vs).cuda().view(torch.float16).view(rows, -1)
    sK[valid] = float("nan")
    sV[valid] = float("inf")
    out = torch.full((B * Hq * Q * D,), float("nan"), dtype=torch.float16, device="cuda")
    ws = torch.zeros(va.gqa_workspace_bytes(B, Hq * Q, D, S), dtype=torch.uint8, device="cuda")
    qd = torch.from_numpy(np.ascontiguousarray(q).ravel()).cuda().view(torch.float16)
    b = va.DeviceBufs(K, V, sK, sV, qd, out, ws)
    for _ in range(2):
        va.decode_multiquery(fmt, b, torch.from_numpy(lens).cuda(), B, Hq, Hkv, Q, Lmax, D, S)
        torch.cuda.synchronize()
        got = out.float().cpu().numpy().reshape(B, Hq, Q, D)
        err = np.abs(got - ref)
        bad = ~(err <= ATOL + RTOL * np.abs(ref))
        assert not bad.any(), f"{case}: {bad.sum()} bad, maxerr {np.nanmax(err):.3e}"
    assert va.device_error() == 0


def test_multiquery_rejects_unsupported(va):
    import torch
    B, Hq, Hkv, Q, Lmax, D = 1, 4, 4, 3, 64, 128  # 3 slots per KV head
    K = torch.zeros(B * Hkv * Lmax * 64, dtype=torch.uint8, device="cuda")
    sK = torch.zeros(B * Hkv * Lmax * 2, dtype=torch.float16, device="cuda")
    q = torch.zeros(B * Hq * Q * D, dtype=torch.float16, device="cuda")
    ws = torch.zeros(va.gqa_workspace_bytes(B, Hq * Q, D, 1), dtype=torch.uint8, device="cuda")
    b = va.DeviceBufs(K, K, sK, sK, q, torch.zeros_like(q), ws)
    with pytest.raises(RuntimeError):
        va.decode_multiquery("q4+", b, torch.full((B,), Lmax, dtype=torch.int32, device="cuda"), B, Hq, Hkv, Q,
                             Lmax, D, 1)
