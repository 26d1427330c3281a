"""GPU parity tests: the sm_100a kernels (called through the C ABI) against the
CPU oracle and the golden vectors made by the reference's own host code.

Tolerance for attention outputs (fp16 out, fp32 math): |got - ref| <=
ATOL + RTOL*|ref| with ATOL = 2e-3, RTOL = 1e-3, checked
against the double-precision reference over the exactly dequantized cache.
Quantizer codes and scales: bit-exact.
"""
import hashlib

import numpy as np
import pytest

from oracle.oracle import BITS, FORMATS, SELFTEST_CASES
from tests.golden.inputs import HASH_CONFIGS, edge_input, hash_config_inputs

pytestmark = pytest.mark.gpu

ATOL, RTOL = 2e-3, 1e-3


def sha(*arrays):
    h = hashlib.sha256()
    for a in arrays:
        h.update(np.ascontiguousarray(a).tobytes())
    return h.hexdigest()


@pytest.fixture(scope="module")
def va():
    import torch
    assert torch.cuda.is_available(), "GPU tests need a CUDA device"
    import voltattn_b200
    return voltattn_b200


def to_dev(a, dtype=None):
    import torch
    t = torch.from_numpy(np.ascontiguousarray(a))
    if dtype is not None:
        t = t.view(dtype)
    return t.cuda()


def upload_case(va, fmt, d, H, L, D, gpu_quantize=True):
    """Device buffers for one case. Quantized formats are packed by the GPU
    quantizer from the fp32 data (checked bit-exact against the oracle)."""
    import torch
    if fmt.startswith("f16"):
        K = to_dev(d["kx"]).half()
        V = to_dev(d["vx"]).half()
        return K, V, None, None
    bits = BITS[fmt]
    if gpu_quantize:
        K, sK = va.quantize(to_dev(d["kx"]), bits, H, L, D)
        V, sV = va.quantize(to_dev(d["vx"]), bits, H, L, D)
        torch.cuda.synchronize()
        assert np.array_equal(K.cpu().numpy(), d["kc"]) and np.array_equal(sK.cpu().view(torch.uint16).numpy(), d["ks"])
        assert np.array_equal(V.cpu().numpy(), d["vc"]) and np.array_equal(sV.cpu().view(torch.uint16).numpy(), d["vs"])
        return K, V, sK, sV
    return (to_dev(d["kc"]), to_dev(d["vc"]), to_dev(d["ks"]).view(torch.float16),
            to_dev(d["vs"]).view(torch.float16))


def run_decode(va, fmt, bufs, q, H, L, D, S, fused=True):
    import torch
    out = torch.full((H * D,), float("nan"), dtype=torch.float16, device="cuda")
    if fused:
        ws = va.new_workspace(H, D, S)
    else:  # the reference's workspace size: decode + separate combine
        ws = torch.empty(H * S * (D + 2), dtype=torch.float32, device="cuda")
    K, V, sK, sV = bufs
    va.launch(fmt, va.DeviceBufs(K, V, sK, sV, q, out, ws), H, L, D, S)
    torch.cuda.synchronize()
    if fused:
        assert int(ws[va.workspace_bytes(H, D, S) - 256:].count_nonzero()) == 0, "counters not reset"
    return out.float().cpu().numpy()


def check_close(got, ref, what):
    err = np.abs(got.astype(np.float64) - ref.astype(np.float64))
    bad = err > ATOL + RTOL * np.abs(ref)
    assert not bad.any(), f"{what}: {bad.sum()} bad, maxerr {err.max():.3e}"
    return err.max()


# ---- quantizer ----------------------------------------------------------------

@pytest.mark.parametrize("bits", [8, 4, 3])
def test_quantizer_edge_cases(va, golden, bits):
    import torch
    H, L, D, x = edge_input()
    c, s = va.quantize(to_dev(x), bits, H, L, D)
    torch.cuda.synchronize()
    e = golden["edge"]
    assert np.array_equal(c.cpu().numpy(), e[f"q{bits}_codes"])
    assert np.array_equal(s.cpu().view(torch.uint16).numpy(), e[f"q{bits}_scales"])


@pytest.mark.parametrize("name", list(HASH_CONFIGS))
def test_quantizer_config_digests(va, oracle, golden, name):
    """Full-size quantizer outputs (incl. the L=16384 bench data) hash equal to
    the reference quantize()'s."""
    import torch
    cfg = HASH_CONFIGS[name]
    H, L, D = cfg["H"], cfg["L"], cfg["D"]
    kx, vx = hash_config_inputs(oracle, name)
    for bits in (8, 4, 3):
        for tag, x in (("k", kx), ("v", vx)):
            c, s = va.quantize(to_dev(x), bits, H, L, D)
            torch.cuda.synchronize()
            assert sha(c.cpu().numpy(), s.cpu().view(torch.uint16).numpy()) == \
                golden["digests"][f"{name}_q{bits}_{tag}_sha"], (bits, tag)


# ---- the 42 selftest cases ---------------------------------------------------------

@pytest.mark.parametrize("fmt", FORMATS)
@pytest.mark.parametrize("case", SELFTEST_CASES, ids=lambda c: "H{}_L{}_D{}_S{}".format(*c))
def test_selftest_case(va, oracle, golden, fmt, case):
    H, L, D, S = case
    d = oracle.case_inputs(fmt, H, L, D, oracle.selftest_seed(H, L, D, S))
    ref = oracle.reference(d["kd"], d["vd"], d["q"], H, L, D)
    tag = f"H{H}_L{L}_D{D}_S{S}"
    gkey = f"{tag}_f16_ref" if fmt.startswith("f16") else f"{tag}_q{BITS[fmt]}_ref"
    assert np.array_equal(ref, golden["selftest"][gkey])
    bufs = upload_case(va, fmt, d, H, L, D)
    q = to_dev(d["q"]).view(__import__("torch").float16)
    check_close(run_decode(va, fmt, bufs, q, H, L, D, S, fused=True), ref, f"{fmt} {tag} fused")
    check_close(run_decode(va, fmt, bufs, q, H, L, D, S, fused=False), ref, f"{fmt} {tag} 2-launch")


# ---- edge shapes ----------------------------------------------------------------------

EDGE_SHAPES = [
    (1, 1, 128, 1), (1, 7, 128, 1), (1, 8, 128, 1), (1, 9, 64, 2), (3, 13, 128, 4),   # tiny / ragged tails
    (5, 100, 64, 100), (2, 300, 128, 64),                                             # S > L/8: empty splits
    (7, 1031, 128, 5), (3, 2049, 64, 3),                                              # odd L, tensor end ragged
    (4, 4096, 128, 1), (1, 20000, 128, 37),                                           # long units
]


@pytest.mark.parametrize("fmt", ["f16+", "q8+", "q4+", "q3+", "f16", "q8", "q4"])
@pytest.mark.parametrize("shape", EDGE_SHAPES, ids=lambda c: "H{}_L{}_D{}_S{}".format(*c))
def test_edge_shapes(va, oracle, fmt, shape):
    import torch
    H, L, D, S = shape
    d = oracle.case_inputs(fmt, H, L, D, 1000 + H * 7 + L + S)
    ref = oracle.reference(d["kd"], d["vd"], d["q"], H, L, D)
    bufs = upload_case(va, fmt, d, H, L, D)
    q = to_dev(d["q"]).view(torch.float16)
    check_close(run_decode(va, fmt, bufs, q, H, L, D, S, fused=True), ref, f"{fmt} {shape}")
    if not fmt.endswith("+"):
        return
    check_close(run_decode(va, fmt, bufs, q, H, L, D, S, fused=False), ref, f"{fmt} {shape} 2-launch")


@pytest.mark.parametrize("fmt", ["f16+", "q8+", "q4+", "q3+"])
def test_neighbour_rows_with_nan_do_not_leak(va, oracle, fmt):
    """Rows of other heads that a tile reads (masked) must not contaminate a
    head even when they hold nan/inf: head 1 is poisoned, heads 0 and 2 are
    checked."""
    import torch
    H, L, D, S = 3, 77, 128, 2
    d = oracle.case_inputs(fmt, H, L, D, 4242)
    ref = oracle.reference(d["kd"], d["vd"], d["q"], H, L, D)
    K, V, sK, sV = upload_case(va, fmt, d, H, L, D, gpu_quantize=False)
    rb = K.numel() // (H * L)
    if fmt.startswith("f16"):
        K.view(H, L, D)[1].fill_(float("nan"))
        V.view(H, L, D)[1].fill_(float("inf"))
    else:
        sK.view(H, L, -1)[1].fill_(float("nan"))
        sV.view(H, L, -1)[1].fill_(float("inf"))
    assert rb > 0
    q = to_dev(d["q"]).view(torch.float16)
    got = run_decode(va, fmt, (K, V, sK, sV), q, H, L, D, S)
    for h in (0, 2):
        check_close(got[h * D:(h + 1) * D], ref[h * D:(h + 1) * D], f"{fmt} head {h}")


def test_outlier_input(va, oracle):
    """Config 4 input: 1 % of K entries scaled x8 (stresses the group scales)."""
    import torch
    from tests.golden.inputs import outlier_mask
    H, L, D, S = 32, 1024, 128, 8
    kx, vx, q = oracle.gen_case(0x0D17EE, H, L, D)
    kx = kx.copy()
    kx[outlier_mask(kx.size, 7)] *= 8.0
    for fmt in ["f16+", "q8+", "q4+", "q3+", "q8", "q4", "f16"]:
        if fmt.startswith("f16"):
            kd, vd = oracle.round_to_half(kx), oracle.round_to_half(vx)
            bufs = (to_dev(kx).half(), to_dev(vx).half(), None, None)
        else:
            bits = BITS[fmt]
            K, sK = va.quantize(to_dev(kx), bits, H, L, D)
            V, sV = va.quantize(to_dev(vx), bits, H, L, D)
            torch.cuda.synchronize()
            kd = oracle.dequant(K.cpu().numpy(), sK.cpu().view(torch.uint16).numpy(), H, L, D, bits)
            vd = oracle.dequant(V.cpu().numpy(), sV.cpu().view(torch.uint16).numpy(), H, L, D, bits)
            bufs = (K, V, sK, sV)
        ref = oracle.reference(kd, vd, q, H, L, D, threads=8)
        check_close(run_decode(va, fmt, bufs, to_dev(q).view(torch.float16), H, L, D, S), ref, fmt)


@pytest.mark.parametrize("fmt", ["f16+", "q8+", "q4+", "q3+"])
def test_headline_size(va, oracle, fmt):
    """BASELINE config 2 at full size (H=32, D=128, L=16384) against the
    double-precision reference, with the suggested split count."""
    import torch
    H, L, D = 32, 16384, 128
    kx, vx, q = oracle.gen_case(0xBEEF, H, L, D)
    if fmt.startswith("f16"):
        kd, vd = oracle.round_to_half(kx), oracle.round_to_half(vx)
        bufs = (to_dev(kx).half(), to_dev(vx).half(), None, None)
    else:
        bits = BITS[fmt]
        K, sK = va.quantize(to_dev(kx), bits, H, L, D)
        V, sV = va.quantize(to_dev(vx), bits, H, L, D)
        torch.cuda.synchronize()
        kd = oracle.dequant(K.cpu().numpy(), sK.cpu().view(torch.uint16).numpy(), H, L, D, bits)
        vd = oracle.dequant(V.cpu().numpy(), sV.cpu().view(torch.uint16).numpy(), H, L, D, bits)
        bufs = (K, V, sK, sV)
    ref = oracle.reference(kd, vd, q, H, L, D, threads=8)
    S = va.suggest_splits(fmt, H, L, D)
    qd = to_dev(q).view(torch.float16)
    check_close(run_decode(va, fmt, bufs, qd, H, L, D, S), ref, f"{fmt} S={S}")
    check_close(run_decode(va, fmt, bufs, qd, H, L, D, 9), ref, f"{fmt} S=9")


# ---- split-L partials + combine (multi-GPU building blocks, on one GPU) -------------

@pytest.mark.parametrize("fmt", ["f16+", "q8+", "q4+", "q3+"])
def test_partials_and_combine(va, oracle, fmt):
    """Split the KV length into R contiguous ranges held as separate caches (as
    R GPUs would), decode each into (m, l, o) partials, merge with
    va_combine_partials, compare with the single-cache reference."""
    import torch
    H, L, D, R = 4, 1000, 128, 3
    d = oracle.case_inputs(fmt, H, L, D, 777)
    ref = oracle.reference(d["kd"], d["vd"], d["q"], H, L, D)
    q = to_dev(d["q"]).view(torch.float16)
    bounds = [0, 333, 334, 1000]
    parts = torch.empty(R, H, 1, D + 2, dtype=torch.float32, device="cuda")
    for r in range(R):
        j0, j1 = bounds[r], bounds[r + 1]
        Lr = j1 - j0
        kx = d["kx"].reshape(H, L, D)[:, j0:j1].copy()
        vx = d["vx"].reshape(H, L, D)[:, j0:j1].copy()
        sub = {"kx": kx.ravel(), "vx": vx.ravel()}
        if not fmt.startswith("f16"):
            bits = BITS[fmt]
            sub["kc"], sub["ks"] = oracle.quantize(kx, H, Lr, D, bits)
            sub["vc"], sub["vs"] = oracle.quantize(vx, H, Lr, D, bits)
        bufs = upload_case(va, fmt, sub, H, Lr, D, gpu_quantize=False)
        S = 2
        ws = va.new_workspace(H, D, S)
        out = torch.empty(H * D, dtype=torch.float16, device="cuda")
        va.decode_partial(fmt, va.DeviceBufs(*bufs, q, out, ws), H, Lr, D, S, parts[r])
    out = torch.empty(H * D, dtype=torch.float16, device="cuda")
    va.combine_partials(parts, R, H, 1, D, out)
    torch.cuda.synchronize()
    # the reference's own quantization differs per range only in which rows a
    # group belongs to (groups are along D), so the dequantized cache is equal
    check_close(out.float().cpu().numpy(), ref, fmt)


# ---- reference kernels rebuilt for sm_100a, same buffers -----------------------------

def test_reference_kernels_agree(va, oracle):
    """The reference's own kernels (oracle/_ref, compiled from its source for
    sm_100a) on the same device buffers agree with ours within tolerance."""
    import os
    import torch
    from oracle.oracle import REF_SO, RefLib
    if not os.path.exists(REF_SO):
        pytest.skip("reference library not built")
    r = RefLib()
    H, L, D, S = 8, 513, 128, 4
    for i, fmt in enumerate(FORMATS):
        d = oracle.case_inputs(fmt, H, L, D, 31337)
        ref = oracle.reference(d["kd"], d["vd"], d["q"], H, L, D)
        K, V, sK, sV = upload_case(va, fmt, d, H, L, D, gpu_quantize=False)
        q = to_dev(d["q"]).view(torch.float16)
        out = torch.empty(H * D, dtype=torch.float16, device="cuda")
        ws = torch.empty(H * S * (D + 2), dtype=torch.float32, device="cuda")
        ptr = lambda t: None if t is None else t.data_ptr()  # noqa: E731
        assert r.lib.ref_launch(i, ptr(K), ptr(V), ptr(sK), ptr(sV), ptr(q), ptr(out), ptr(ws), H, L, D, S, 1) == 0
        theirs = out.float().cpu().numpy()
        check_close(theirs, ref, f"reference {fmt}")
        ours = run_decode(va, fmt, (K, V, sK, sV), q, H, L, D, S)
        check_close(ours, theirs.astype(np.float64), f"ours vs reference kernels {fmt}")


# ---- probe and device error word ------------------------------------------------------

def test_probe_ceiling(va):
    g0 = va.probe_ceiling(0, nbytes=1 << 30, reps=5, method=0)
    g1 = va.probe_ceiling(0, nbytes=1 << 30, reps=5, method=1)
    for g in (g0, g1):
        assert 1000.0 < g < 20000.0, g


def test_no_device_errors(va):
    assert va.device_error() == 0
