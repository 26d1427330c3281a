"""Pins the CPU oracle (oracle/voltattn_oracle.cpp) to golden vectors made by
the reference's own host functions (tests/golden/make_golden.py)."""
import hashlib

import numpy as np
import pytest

from oracle.oracle import SELFTEST_CASES
from tests.golden.inputs import HASH_CONFIGS, edge_input, half_patterns, hash_config_inputs


def sha(*arrays):
    h = hashlib.sha256()
    for a in arrays:
        h.update(np.ascontiguousarray(a).tobytes())
    return h.hexdigest()


def test_half_conversions(oracle, golden):
    d = golden["digests"]
    assert sha(oracle.f2h(half_patterns())) == d["f2h_sha"]
    hall = np.arange(65536, dtype=np.uint32).astype(np.uint16)
    assert sha(oracle.h2f(hall)) == d["h2f_sha"]


@pytest.mark.parametrize("case", SELFTEST_CASES, ids=lambda c: "H{}_L{}_D{}_S{}".format(*c))
def test_selftest_case(oracle, golden, case):
    H, L, D, S = case
    tag = f"H{H}_L{L}_D{D}_S{S}"
    g = golden["selftest"]
    kx, vx, q = oracle.gen_case(oracle.selftest_seed(H, L, D, S), H, L, D)
    assert np.array_equal(q, g[f"{tag}_q"])
    ref = oracle.reference(oracle.round_to_half(kx), oracle.round_to_half(vx), q, H, L, D)
    assert np.array_equal(ref.view(np.uint32), g[f"{tag}_f16_ref"].view(np.uint32))
    for bits in (8, 4, 3):
        kc, ks = oracle.quantize(kx, H, L, D, bits)
        vc, vs = oracle.quantize(vx, H, L, D, bits)
        assert sha(kc, ks, vc, vs) == golden["digests"][f"{tag}_q{bits}_sha"], bits
        if f"{tag}_q{bits}_kcodes" in g:
            assert np.array_equal(kc, g[f"{tag}_q{bits}_kcodes"])
            assert np.array_equal(ks, g[f"{tag}_q{bits}_kscales"])
        kd = oracle.dequant(kc, ks, H, L, D, bits)
        vd = oracle.dequant(vc, vs, H, L, D, bits)
        out = oracle.reference(kd, vd, q, H, L, D)
        assert np.array_equal(out.view(np.uint32), g[f"{tag}_q{bits}_ref"].view(np.uint32)), bits
        # threaded variant is the same math
        out4 = oracle.reference(kd, vd, q, H, L, D, threads=4)
        assert np.array_equal(out, out4)


@pytest.mark.parametrize("bits", [8, 4, 3])
def test_edge_quantizer(oracle, golden, bits):
    e = golden["edge"]
    H, L, D, x = edge_input()
    assert np.array_equal(x.view(np.uint32), e["x"].view(np.uint32))
    c, s = oracle.quantize(x, H, L, D, bits)
    assert np.array_equal(c, e[f"q{bits}_codes"])
    assert np.array_equal(s, e[f"q{bits}_scales"])


@pytest.mark.parametrize("name", [k for k in HASH_CONFIGS if HASH_CONFIGS[k]["L"] <= 4096])
def test_config_digests(oracle, golden, name):
    cfg = HASH_CONFIGS[name]
    H, L, D = cfg["H"], cfg["L"], cfg["D"]
    kx, vx = hash_config_inputs(oracle, name)
    for bits in (8, 4, 3):
        assert sha(*oracle.quantize(kx, H, L, D, bits)) == golden["digests"][f"{name}_q{bits}_k_sha"]
        assert sha(*oracle.quantize(vx, H, L, D, bits)) == golden["digests"][f"{name}_q{bits}_v_sha"]


def test_combine_matches_reference_softmax(oracle):
    """Split partials merged by the LSE combine equal the one-pass reference."""
    H, L, D, S = 3, 301, 64, 4
    kx, vx, q = oracle.gen_case(99, H, L, D)
    kd, vd = oracle.round_to_half(kx), oracle.round_to_half(vx)
    chunk = -(-L // S)
    ws = np.concatenate([oracle.partial(kd, vd, q, H, L, D, h, s * chunk, min(L, (s + 1) * chunk))
                         for h in range(H) for s in range(S)])
    out = oracle.h2f(oracle.combine(ws, H, S, D))
    ref = oracle.reference(kd, vd, q, H, L, D)
    np.testing.assert_allclose(out, ref, atol=1e-3, rtol=1e-3)
