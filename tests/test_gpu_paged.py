"""Paged KV cache: va_decode_paged against the oracle's GQA restatement over
the same logical cache, and va_append_kv_paged against the quantizer. The pool
holds the sequences' pages in a random order among unused pages whose scales
are nan (and rows past lens[b] inside a sequence's last page likewise), so a
wrong page or an unmasked row shows up in the output. No reference
counterpart: the reference is a single contiguous batch-1 cache."""
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


def make_table(rng, lens, Lmax, page_rows, spare):
    """Random block table: each sequence's pages at shuffled pool indices,
    `spare` pool pages unused, -1 past a sequence's last page."""
    need = [(int(l) + page_rows - 1) // page_rows for l in lens]
    max_pages = (Lmax + page_rows - 1) // page_rows
    num_pages = sum(need) + spare
    perm = rng.permutation(num_pages)
    table = np.full((len(lens), max_pages), -1, np.int32)
    k = 0
    for b, n in enumerate(need):
        table[b, :n] = perm[k:k + n]
        k += n
    return table, max_pages, num_pages


def build_pool(rng, codes, scales, lens, table, num_pages, Hkv, Lmax, D, bits, page_rows, fill_scale):
    """Scatter a contiguous [B][Hkv][Lmax] cache into the page pool; unused
    rows get random codes and `fill_scale` scales."""
    B = len(lens)
    rb, ng = D * bits // 8, D // 64
    pc = rng.integers(0, 256, size=(num_pages, Hkv, page_rows, rb), dtype=np.uint8)
    ps = np.full((num_pages, Hkv, page_rows, ng), np.float16(fill_scale)).view(np.uint16)
    c3 = codes.reshape(B, Hkv, Lmax, rb)
    s3 = scales.reshape(B, Hkv, Lmax, ng)
    for b in range(B):
        for j in range(table.shape[1]):
            pg = table[b, j]
            if pg < 0:
                continue
            r0, r1 = j * page_rows, min((j + 1) * page_rows, int(lens[b]))
            pc[pg, :, :r1 - r0] = c3[b, :, r0:r1]
            ps[pg, :, :r1 - r0] = s3[b, :, r0:r1]
    return pc.reshape(-1), ps.reshape(-1)


CASES = [  # fmt, B, Hq, Hkv, Lmax, page_rows, S
    ("q4+", 3, 8, 2, 700, 64, 3),
    ("q4+", 2, 16, 4, 1031, 256, 2),
    ("q4+", 4, 4, 4, 600, 32, 2),
    ("q8+", 3, 4, 4, 777, 96, 3),
    ("q8+", 2, 2, 2, 300, 32, 1),
    ("q4+", 1, 32, 8, 4100, 128, 4),
    ("q4+", 2, 16, 2, 900, 64, 2),   # 8 query heads per KV head
    ("q4+", 2, 8, 4, 500, 32, 2),    # 2 query heads per KV head
    ("q3+", 3, 4, 4, 777, 96, 3),
    ("q3+", 2, 2, 2, 1500, 32, 4),
    # the streaming / grouped-query kernels (page rows a multiple of 8)
    ("f16+", 3, 8, 2, 700, 64, 3),
    ("bf16+", 2, 4, 4, 500, 24, 2),
    ("f8+", 2, 8, 4, 900, 40, 3),
    ("q8+", 2, 16, 4, 1031, 64, 2),   # 4 query heads per KV head
    ("q3+", 3, 8, 2, 777, 96, 3),     # 4 query heads per KV head
    ("q4+", 2, 4, 4, 600, 16, 2),     # pages too small for the tile kernel
    ("q4+", 2, 8, 4, 700, 32, 2, 64),  # D = 64
    ("q8+", 1, 2, 2, 333, 8, 1, 64),
]


def _encode(oracle, x, rows, D, fmt):
    """codes (uint8 rows), scales (uint16, or None) and the exactly decoded
    values of x in fmt, by the oracle."""
    if fmt == "f16+":
        h = oracle.f2h(x)
        return h.view(np.uint8), None, oracle.h2f(h)
    if fmt == "bf16+":
        b = oracle.f2bf(x)
        return b.view(np.uint8), None, (b.astype(np.uint32) << 16).view(np.float32)
    if fmt == "f8+":
        c, s = oracle.quantize_f8(x, 1, rows, D)
        return c, s, oracle.dequant_f8(c, s, 1, rows, D)
    bits = BITS[fmt]
    c, s = oracle.quantize(x, 1, rows, D, bits)
    return c, s, oracle.dequant(c, s, 1, rows, D, bits)


@pytest.mark.parametrize("case", CASES, ids=lambda c: "{}_B{}_Hq{}_Hkv{}_L{}_P{}_S{}".format(*c[:7])
                         + ("_D{}".format(c[7]) if len(c) > 7 else ""))
def test_decode_paged(va, oracle, case):
    import torch
    fmt, B, Hq, Hkv, Lmax, page_rows, S = case[:7]
    D = case[7] if len(case) > 7 else 128
    bits = {"f16+": 16, "bf16+": 16, "f8+": 8}.get(fmt) or BITS[fmt]
    rng = np.random.default_rng(B * 7919 + Hq * 31 + Lmax + page_rows + D)
    lens = rng.integers(1, Lmax + 1, size=B).astype(np.int32)
    lens[0] = Lmax
    rows = B * Hkv * Lmax
    kx, vx, _ = oracle.gen_case(int(rng.integers(1 << 30)), 1, rows, D)
    q = oracle.f2h(rng.standard_normal(B * Hq * D).astype(np.float32))
    kc, ks, kd = _encode(oracle, kx, rows, D, fmt)
    vc, vs, vd = _encode(oracle, vx, rows, D, fmt)
    ref = oracle.reference_gqa(kd, vd, q, lens, B, Hq, Hkv, Lmax, D)
    table, max_pages, num_pages = make_table(rng, lens, Lmax, page_rows, 5)
    if ks is None:  # no scales: unused rows hold random bit patterns (nan and inf among them)
        pkc, _ = build_pool(rng, kc, np.zeros(rows * (D // 64), np.uint16), lens, table, num_pages, Hkv, Lmax, D,
                            bits, page_rows, 0.0)
        pvc, _ = build_pool(rng, vc, np.zeros(rows * (D // 64), np.uint16), lens, table, num_pages, Hkv, Lmax, D,
                            bits, page_rows, 0.0)
        pks = pvs = None
    else:
        pkc, pks = build_pool(rng, kc, ks, lens, table, num_pages, Hkv, Lmax, D, bits, page_rows, np.nan)
        pvc, pvs = build_pool(rng, vc, vs, lens, table, num_pages, Hkv, Lmax, D, bits, page_rows, np.inf)
    K, V = torch.from_numpy(pkc).cuda(), torch.from_numpy(pvc).cuda()
    sK = None if pks is None else torch.from_numpy(pks).cuda().view(torch.float16)
    sV = None if pvs is None else torch.from_numpy(pvs).cuda().view(torch.float16)
    qd = torch.from_numpy(q).cuda().view(torch.float16)
    out = torch.full((B * Hq * D,), float("nan"), dtype=torch.float16, device="cuda")
    ws = torch.zeros(va.gqa_workspace_bytes(B, Hq, D, S), dtype=torch.uint8, device="cuda")
    bt = torch.from_numpy(table).cuda()
    lens_d = torch.from_numpy(lens).cuda()
    for _ in range(2):  # the second call reuses the workspace
        va.decode_paged(fmt, va.DeviceBufs(K, V, sK, sV, qd, out, ws), bt, max_pages, lens_d, B, Hq, Hkv,
                        page_rows, num_pages, D, S)
        torch.cuda.synchronize()
        got = out.float().cpu().numpy()
        err = np.abs(got - ref)
        bad = ~(err <= ATOL + RTOL * np.abs(ref))
        assert not bad.any(), f"{case}: {bad.sum()} bad, maxerr {np.nanmax(err):.3e}"
    assert va.device_error() == 0


@pytest.mark.parametrize("bits", [8, 4, 3])
def test_append_paged_matches_quantizer(va, oracle, bits):
    import torch
    B, Hkv, D, page_rows, max_pages = 3, 2, 128, 64, 4
    num_pages = B * max_pages + 2
    rng = np.random.default_rng(bits)
    table = rng.permutation(num_pages)[:B * max_pages].reshape(B, max_pages).astype(np.int32)
    rb, ng = D * bits // 8, D // 64
    codes = torch.zeros(num_pages * Hkv * page_rows * rb, dtype=torch.uint8, device="cuda")
    scales = torch.zeros(num_pages * Hkv * page_rows * ng, dtype=torch.float16, device="cuda")
    pos = np.array([0, 77, 255], np.int32)
    x = rng.standard_normal(B * Hkv * D).astype(np.float32) * 3
    va.append_kv_paged(torch.from_numpy(x).cuda(), bits, codes, scales, torch.from_numpy(table).cuda(), max_pages, B,
                       Hkv, page_rows, num_pages, D, torch.from_numpy(pos).cuda())
    torch.cuda.synchronize()
    want_c, want_s = oracle.quantize(x, 1, B * Hkv, D, bits)
    pc = codes.cpu().numpy().reshape(num_pages, Hkv, page_rows, rb)
    ps = scales.cpu().view(torch.uint16).numpy().reshape(num_pages, Hkv, page_rows, ng)
    wc, ws_ = want_c.reshape(B, Hkv, rb), want_s.reshape(B, Hkv, ng)
    for b in range(B):
        pg = table[b, pos[b] // page_rows]
        r = pos[b] % page_rows
        assert (pc[pg, :, r] == wc[b]).all()
        assert (ps[pg, :, r] == ws_[b]).all()
    # nothing else was written
    assert int((pc != 0).sum()) == int((wc != 0).sum())


def test_paged_rejects_unsupported(va):
    import torch
    B, Hq, Hkv, D, page_rows, max_pages, num_pages = 1, 4, 4, 128, 16, 4, 4
    dev = "cuda"
    K = torch.zeros(num_pages * Hkv * page_rows * 64, dtype=torch.uint8, device=dev)
    sK = torch.zeros(num_pages * Hkv * page_rows * 2, dtype=torch.float16, device=dev)
    q = torch.zeros(B * Hq * D, dtype=torch.float16, device=dev)
    out = torch.zeros_like(q)
    ws = torch.zeros(va.gqa_workspace_bytes(B, Hq, D, 1), dtype=torch.uint8, device=dev)
    bt = torch.zeros(B * max_pages, dtype=torch.int32, device=dev)
    lens = torch.ones(B, dtype=torch.int32, device=dev)
    b = va.DeviceBufs(K, K, sK, sK, q, out, ws)
    with pytest.raises(RuntimeError):  # page rows not a multiple of 8
        va.decode_paged("q4+", b, bt, max_pages, lens, B, Hq, Hkv, 12, num_pages, D, 1)
    with pytest.raises(RuntimeError):  # q4c+: one query head per KV head only
        va.decode_paged("q4c+", b, bt, max_pages, lens, B, 2 * Hkv, Hkv, 32, num_pages, D, 1)
    with pytest.raises(RuntimeError):  # 3 query heads per KV head
        va.decode_paged("q8+", b, bt, max_pages, lens, B, 3 * Hkv, Hkv, 32, num_pages, D, 1)
