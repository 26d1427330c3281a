"""q4c+ (per-channel K scales, per-token V scales; no reference counterpart):
the GPU quantizers are bit-exact with the oracle's (same group rule as the
reference's quantize, with a channel over all positions or a whole row as the
group), and the tile kernel's decode matches the double-precision reference over
the exactly dequantized cache."""
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


def outlier_input(H, L, D, seed, edge=True):
    rng = np.random.default_rng(seed)
    x = rng.standard_normal((H, L, D)).astype(np.float32)
    x[:, :, rng.integers(0, D, 4)] *= 20.0          # outlier channels, the case per-channel K serves
    if edge:  # quantizer edge values (an inf makes its whole channel's scale inf)
        x[0, 3, :8] = [np.inf, -np.inf, np.nan, 0.0, 1e30, -1e-30, 7.0, -7.0]
    x[1 % H, :, 5] = 0.0                             # an all-zero channel: scale 1
    return x.ravel()


@pytest.mark.parametrize("bits", [8, 4])
@pytest.mark.parametrize("D", [128, 64])
def test_quantizers_bit_exact(va, oracle, bits, D):
    import torch
    H, L = 3, 333
    x = outlier_input(H, L, D, bits * 100 + D)
    xd = torch.from_numpy(x).cuda()
    for gpu_fn, ora_fn in ((va.quantize_kchan, oracle.quantize_kchan), (va.quantize_vtok, oracle.quantize_vtok)):
        codes, scales = gpu_fn(xd, bits, H, L, D)
        torch.cuda.synchronize()
        wc, ws = ora_fn(x, H, L, D, bits)
        assert (scales.cpu().view(torch.uint16).numpy() == ws).all(), gpu_fn.__name__
        assert (codes.cpu().numpy() == wc).all(), gpu_fn.__name__


@pytest.mark.parametrize("case", [(8, 257, 3), (3, 13, 4), (7, 1031, 5), (2, 4096, 9), (32, 2048, 3), (5, 600, 40)],
                         ids=lambda c: "H{}_L{}_S{}".format(*c))
def test_decode_q4c(va, oracle, case):
    import torch
    H, L, S = case
    D = 128
    kx = outlier_input(H, L, D, H * 7 + L, edge=False)
    vx = np.random.default_rng(L).standard_normal(H * L * D).astype(np.float32)
    kc, ks = oracle.quantize_kchan(kx, H, L, D, 4)
    vc, vs = oracle.quantize_vtok(vx, H, L, D, 4)
    kd = oracle.dequant_kchan(kc, ks, H, L, D, 4)
    vd = oracle.dequant_vtok(vc, vs, H, L, D, 4)
    q = oracle.f2h(np.random.default_rng(H + L).standard_normal(H * D).astype(np.float32))
    ref = oracle.reference(kd, vd, q, H, L, D)
    K, V = torch.from_numpy(kc).cuda(), torch.from_numpy(vc).cuda()
    sK = torch.from_numpy(ks).cuda().view(torch.float16)
    sV = torch.from_numpy(vs).cuda().view(torch.float16)
    out = va.decode("q4c+", K, V, sK, sV, torch.from_numpy(q).cuda().view(torch.float16), H, L, D, S)
    torch.cuda.synchronize()
    err = np.abs(out.float().cpu().numpy() - ref)
    bad = ~(err <= ATOL + RTOL * np.abs(ref))
    assert not bad.any(), f"{case}: {bad.sum()} bad, maxerr {err.max():.3e}"
    assert va.device_error() == 0


def test_q4c_rejects(va):
    import torch
    H, L, D, S = 2, 64, 64, 1
    K = torch.zeros(H * L * D // 2, dtype=torch.uint8, device="cuda")
    sK = torch.zeros(H * D, dtype=torch.float16, device="cuda")
    sV = torch.zeros(H * L, dtype=torch.float16, device="cuda")
    q = torch.zeros(H * D, dtype=torch.float16, device="cuda")
    with pytest.raises(RuntimeError):  # D = 64: no kernel
        va.decode("q4c+", K, K, sK, sV, q, H, L, D, S)
    D = 128
    q = torch.zeros(H * D, dtype=torch.float16, device="cuda")
    with pytest.raises(RuntimeError):  # slots-only workspace (two-launch mode): not supported
        va.decode("q4c+", K, K, sK, sV, q, H, L, D, S, ws=torch.zeros(H * S * (D + 2), dtype=torch.float32,
                                                                          device="cuda"))


@pytest.mark.parametrize("paged", [False, True], ids=["batched", "paged"])
def test_decode_q4c_batched_and_paged(va, oracle, paged):
    """q4c+ over a batch of sequences with their own lengths (one query head
    per KV head), contiguous [B][Hkv][Lmax] or in a page pool (V row scales
    paged with the rows, K channel scales per sequence and KV head); unused
    pool rows carry nan V scales."""
    import torch
    B, Hkv, Lmax, D, S, P = 3, 4, 700, 128, 3, 64
    rng = np.random.default_rng(11 + paged)
    lens = rng.integers(1, Lmax + 1, size=B).astype(np.int32)
    lens[0] = Lmax
    streams = B * Hkv
    kx = outlier_input(streams, Lmax, D, 5, edge=False)
    vx = rng.standard_normal(streams * Lmax * D).astype(np.float32)
    kc, ks = oracle.quantize_kchan(kx, streams, Lmax, D, 4)
    vc, vs = oracle.quantize_vtok(vx, streams, Lmax, D, 4)
    kd = oracle.dequant_kchan(kc, ks, streams, Lmax, D, 4)
    vd = oracle.dequant_vtok(vc, vs, streams, Lmax, D, 4)
    q = oracle.f2h(rng.standard_normal(B * Hkv * D).astype(np.float32))
    ref = oracle.reference_gqa(kd, vd, q, lens, B, Hkv, Hkv, Lmax, D)
    dev = lambda a: torch.from_numpy(np.ascontiguousarray(a)).cuda()  # noqa: E731
    qd = dev(q).view(torch.float16)
    out = torch.full((B * Hkv * D,), float("nan"), dtype=torch.float16, device="cuda")
    ws = torch.zeros(va.gqa_workspace_bytes(B, Hkv, D, S), dtype=torch.uint8, device="cuda")
    if not paged:
        b = va.DeviceBufs(dev(kc), dev(vc), dev(ks).view(torch.float16), dev(vs).view(torch.float16), qd, out, ws)
        va.decode_gqa("q4c+", b, dev(lens), B, Hkv, Hkv, Lmax, D, S)
    else:
        max_pages = (Lmax + P - 1) // P
        need = [(int(l) + P - 1) // P for l in lens]
        num_pages = sum(need) + 3
        perm = rng.permutation(num_pages)
        table = np.zeros((B, max_pages), np.int32)
        pk = rng.integers(0, 256, size=(num_pages, Hkv, P, D // 2), dtype=np.uint8)
        pv = rng.integers(0, 256, size=(num_pages, Hkv, P, D // 2), dtype=np.uint8)
        psv = np.full((num_pages, Hkv, P), np.float16(np.nan)).view(np.uint16)
        k3, v3 = kc.reshape(B, Hkv, Lmax, D // 2), vc.reshape(B, Hkv, Lmax, D // 2)
        s3 = vs.reshape(B, Hkv, Lmax)
        i = 0
        for bb in range(B):
            for j in range(need[bb]):
                pg = perm[i]
                i += 1
                table[bb, j] = pg
                r0, r1 = j * P, min((j + 1) * P, int(lens[bb]))
                pk[pg, :, :r1 - r0] = k3[bb, :, r0:r1]
                pv[pg, :, :r1 - r0] = v3[bb, :, r0:r1]
                psv[pg, :, :r1 - r0] = s3[bb, :, r0:r1]
        b = va.DeviceBufs(dev(pk.ravel()), dev(pv.ravel()), dev(ks).view(torch.float16),
                          dev(psv.ravel()).view(torch.float16), qd, out, ws)
        va.decode_paged("q4c+", b, dev(table), max_pages, dev(lens), B, Hkv, Hkv, P, num_pages, D, S)
    torch.cuda.synchronize()
    err = np.abs(out.float().cpu().numpy() - ref)
    bad = ~(err <= ATOL + RTOL * np.abs(ref))
    assert not bad.any(), f"{bad.sum()} bad, maxerr {np.nanmax(err):.3e}"
