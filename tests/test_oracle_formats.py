"""The oracle's fp8 (e4m3) and bf16 encoders, checked against the formats'
definitions (no reference counterpart: f8+ and bf16+ are this project's
formats). e4m3: 1 sign, 4 exponent bits with bias 7, 3 mantissa bits, no
infinities, S.1111.111 is nan, largest finite 448; encoding rounds to nearest
even and saturates. bf16: the upper half of an fp32, rounded to nearest even."""
import numpy as np
import pytest


def test_e4m3_decode_table(oracle):
    d = oracle.e4m3_decode(np.arange(256, dtype=np.uint8))
    for code, want in [(0x00, 0.0), (0x01, 2.0 ** -9), (0x07, 7 * 2.0 ** -9), (0x08, 2.0 ** -6), (0x38, 1.0),
                       (0x39, 1.125), (0x3F, 1.875), (0x40, 2.0), (0x7E, 448.0), (0xB8, -1.0), (0xFE, -448.0)]:
        assert d[code] == want, hex(code)
    assert np.isnan(d[0x7F]) and np.isnan(d[0xFF])
    assert np.count_nonzero(np.isnan(d)) == 2
    # every finite code encodes back to itself (-0 included)
    fin = np.flatnonzero(~np.isnan(d)).astype(np.uint8)
    assert (oracle.e4m3_encode(d[fin]) == fin).all()


def test_e4m3_rounding_and_saturation(oracle):
    step = 2.0 ** -9
    cases = [
        (1.0 + 1 / 16, 0x38),        # halfway 1.0 / 1.125 -> even (1.0)
        (1.0 + 3 / 16, 0x3A),        # halfway 1.125 / 1.25 -> even (1.25)
        (1.5 * step, 0x02),          # subnormal halfway 1 / 2 steps -> 2
        (2.5 * step, 0x02),          # 2 / 3 steps -> 2
        (7.5 * step, 0x08),          # rounds up into the smallest normal
        (447.9, 0x7E), (456.0, 0x7E), (464.0, 0x7E), (465.0, 0x7E), (1e6, 0x7E), (np.inf, 0x7E),
        (-np.inf, 0xFE), (-0.0, 0x80), (np.nan, 0x7F),
        (2.0 ** -12, 0x00),          # below half a subnormal step
    ]
    x = np.array([c[0] for c in cases], np.float32)
    got = oracle.e4m3_encode(x)
    for (v, want), g in zip(cases, got):
        assert g == want, (v, hex(g), hex(want))


def test_bf16_rounding_matches_torch(oracle):
    torch = pytest.importorskip("torch")
    rng = np.random.default_rng(5)
    x = np.concatenate([rng.standard_normal(100000).astype(np.float32) * 10,
                        np.array([1.0 + 2 ** -8, 1.0 + 3 * 2 ** -8, 3.4e38, -3.4e38, 1e-40, 0.0, -0.0, np.inf],
                                 np.float32)])
    ours = oracle.f2bf(x)
    theirs = torch.from_numpy(x).to(torch.bfloat16).view(torch.int16).numpy().view(np.uint16)
    assert (ours == theirs).all()
    assert ours[-8] == 0x3F80 and ours[-7] == 0x3F82
