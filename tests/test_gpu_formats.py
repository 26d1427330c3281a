"""bf16+ and f8+ (no reference counterpart): the GPU fp8 group quantizer is
bit-exact with the oracle's (tests/test_oracle_formats.py pins its e4m3
encoder to the format's definition), and batch-1 and grouped-query decodes
match the oracle's double-precision reference over the exactly decoded cache."""
import numpy as np
import pytest

pytestmark = pytest.mark.gpu

ATOL, RTOL = 2e-3, 1e-3


@pytest.fixture(scope="module")
def va():
    import torch
    assert torch.cuda.is_available()
    import voltattn_b200
    return voltattn_b200


def f8_edge_input(H, L, D, seed):
    rng = np.random.default_rng(seed)
    x = (rng.standard_normal(H * L * D) * 3).astype(np.float32)
    g = x.reshape(-1, 64)
    g[0] = 0.0                                        # zero group: scale 1, codes 0
    g[1, :8] = [np.inf, -np.inf, np.nan, 1e30, -1e-30, 448.0, 0.5, -0.5]
    g[2] = np.linspace(-1, 1, 64, dtype=np.float32) * 1e-4
    g[3, ::2] = 1000.0                               # saturating neighbours of the amax
    g[4] = np.float32(65504.0) * np.sign(g[4])       # scale at the fp16 maximum
    return x


@pytest.mark.parametrize("D", [128, 64])
def test_quantize_f8_bit_exact(va, oracle, D):
    import torch
    H, L = 3, 37
    x = f8_edge_input(H, L, D, D)
    codes, scales = va.quantize_f8(torch.from_numpy(x).cuda(), H, L, D)
    torch.cuda.synchronize()
    wc, ws = oracle.quantize_f8(x, H, L, D)
    gc = codes.cpu().numpy()
    gs = scales.cpu().view(torch.uint16).numpy()
    assert (gs == ws).all()
    # nan codes may differ only in the sign bit
    nan = (wc & 0x7F) == 0x7F
    assert (gc[~nan] == wc[~nan]).all(), f"{int((gc[~nan] != wc[~nan]).sum())} codes differ"
    assert ((gc[nan] & 0x7F) == 0x7F).all()


def make_cache(oracle, fmt, x, H, L, D):
    """Codes / scales on the GPU and the exactly decoded fp32 values."""
    import torch
    if fmt == "bf16+":
        bits = oracle.f2bf(x)
        vals = (bits.astype(np.uint32) << 16).view(np.float32)
        return torch.from_numpy(bits.view(np.int16)).cuda(), None, vals
    codes, scales = oracle.quantize_f8(x, H, L, D)
    vals = oracle.dequant_f8(codes, scales, H, L, D)
    return torch.from_numpy(codes).cuda(), torch.from_numpy(scales).cuda().view(torch.float16), vals


CASES = [(8, 257, 128, 3), (3, 13, 128, 4), (5, 100, 64, 100), (7, 1031, 128, 5), (2, 4096, 128, 9),
         (4, 513, 64, 2)]


@pytest.mark.parametrize("fmt", ["bf16+", "f8+"])
@pytest.mark.parametrize("case", CASES, ids=lambda c: "H{}_L{}_D{}_S{}".format(*c))
def test_decode_new_formats(va, oracle, fmt, case):
    import torch
    H, L, D, S = case
    kx, vx, q = oracle.gen_case(H * 131 + L, H, L, D)
    K, sK, kd = make_cache(oracle, fmt, kx, H, L, D)
    V, sV, vd = make_cache(oracle, fmt, vx, H, L, D)
    ref = oracle.reference(kd, vd, q, H, L, D)
    qd = torch.from_numpy(q).cuda().view(torch.float16)
    for fused in (True, False):
        # a workspace of exactly H*S*(D+2) floats selects the two-launch path
        ws = None if fused else torch.zeros(H * S * (D + 2), dtype=torch.float32, device="cuda")
        out = va.decode(fmt, K, V, sK, sV, qd, H, L, D, S, ws=ws)
        torch.cuda.synchronize()
        err = np.abs(out.float().cpu().numpy() - ref)
        bad = ~(err <= ATOL + RTOL * np.abs(ref))
        assert not bad.any(), f"{fmt} {case} fused={fused}: {bad.sum()} bad, maxerr {err.max():.3e}"
    assert va.device_error() == 0


@pytest.mark.parametrize("fmt", ["bf16+", "f8+"])
@pytest.mark.parametrize("case", [(3, 8, 2, 300, 128, 3), (2, 16, 2, 200, 64, 2), (4, 8, 8, 150, 128, 1)],
                         ids=lambda c: "B{}_Hq{}_Hkv{}_L{}_D{}_S{}".format(*c))
def test_gqa_new_formats(va, oracle, fmt, case):
    import torch
    B, Hq, Hkv, Lmax, D, S = case
    rng = np.random.default_rng(B * 100 + Hq + Lmax)
    lens = rng.integers(1, Lmax + 1, size=B).astype(np.int32)
    rows = B * Hkv * Lmax
    kx, vx, _ = oracle.gen_case(int(rng.integers(1 << 30)), 1, rows, D)
    qh = oracle.f2h(rng.standard_normal(B * Hq * D).astype(np.float32))
    K, sK, kd = make_cache(oracle, fmt, kx, 1, rows, D)
    V, sV, vd = make_cache(oracle, fmt, vx, 1, rows, D)
    ref = oracle.reference_gqa(kd, vd, qh, lens, B, Hq, Hkv, Lmax, D)
    out = torch.empty(B * Hq * D, dtype=torch.float16, device="cuda")
    ws = torch.zeros(va.gqa_workspace_bytes(B, Hq, D, S), dtype=torch.uint8, device="cuda")
    b = va.DeviceBufs(K, V, sK, sV, torch.from_numpy(qh).cuda().view(torch.float16), out, ws)
    va.decode_gqa(fmt, b, torch.from_numpy(lens).cuda(), B, Hq, Hkv, Lmax, D, S)
    torch.cuda.synchronize()
    err = np.abs(out.float().cpu().numpy() - ref)
    bad = ~(err <= ATOL + RTOL * np.abs(ref))
    assert not bad.any(), f"{fmt} {case}: {bad.sum()} bad, maxerr {err.max():.3e}"
    assert va.device_error() == 0
