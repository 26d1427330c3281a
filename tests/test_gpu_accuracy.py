"""the quantization error itself. H=32, D=128, L=4096,
q/K/V N(0,1) from the reference's selftest generator (mt19937 normal order,
src/voltattn.cu:839-846); the q8+ (and q4+, q3+) decodes on the GPU against
the fp16 attention output: the double-precision reference over the
fp16-rounded cache. The reference's run_case keeps this error out of its
pass gate (it compares against the dequantized cache); here it is measured
and bounded, and the figures are printed (pytest -s)."""
import numpy as np
import pytest

from oracle.oracle import BITS

pytestmark = pytest.mark.gpu

# Bounds on max |quantized - fp16 attention|: the measured error times ~3
BOUND = {"q8+": 0.02, "q4+": 0.2, "q3+": 0.5}


@pytest.fixture(scope="module")
def va():
    import torch
    assert torch.cuda.is_available()
    import voltattn_b200
    return voltattn_b200


def test_config1_quantization_error(va, oracle):
    import torch
    H, L, D = 32, 4096, 128
    kx, vx, q = oracle.gen_case(20260, H, L, D)
    ref = oracle.reference(oracle.round_to_half(kx), oracle.round_to_half(vx), q, H, L, D, threads=8)
    qd = torch.from_numpy(q).cuda().view(torch.float16)
    f16 = va.decode("f16+", torch.from_numpy(kx).cuda().half(), torch.from_numpy(vx).cuda().half(), None, None, qd,
                    H, L, D).float().cpu().numpy()
    err16 = np.abs(f16 - ref)
    assert (err16 <= 2e-3 + 1e-3 * np.abs(ref)).all(), err16.max()
    print(f"\nconfig 1 (H={H} L={L} D={D}): |ref| mean {np.abs(ref).mean():.4f}; f16+ max err {err16.max():.2e}")
    for fmt in ("q8+", "q4+", "q3+"):
        bits = BITS[fmt]
        K, sK = va.quantize(torch.from_numpy(kx).cuda(), bits, H, L, D)
        V, sV = va.quantize(torch.from_numpy(vx).cuda(), bits, H, L, D)
        got = va.decode(fmt, K, V, sK, sV, qd, H, L, D).float().cpu().numpy()
        err = np.abs(got - ref)
        print(f"{fmt} vs fp16 attention: max {err.max():.3e} mean {err.mean():.3e}")
        assert err.max() < BOUND[fmt], (fmt, err.max())
    assert va.device_error() == 0
