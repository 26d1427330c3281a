"""Parity run for one decode consumer, selected by VOLTATTN_CONSUMER (read once
per process, hence a separate process per consumer; driven by
tests/test_gpu_consumers.py). Exits non-zero on the first mismatch."""
import os
import sys

import numpy as np

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
sys.path.insert(0, ROOT)


def main():
    import torch
    import voltattn_b200 as va
    from oracle.oracle import BITS, Oracle
    o = Oracle()
    ATOL, RTOL = 2e-3, 1e-3
    fails = 0
    # batch-1 multi-head: ragged tails, empty splits, D=64/128
    for fmt in ["q8+", "q4+", "q3+"]:
        for (H, L, D, S) in [(8, 257, 128, 3), (3, 13, 128, 4), (5, 100, 64, 100), (7, 1031, 128, 5),
                             (8, 513, 64, 4), (2, 4096, 128, 5)]:
            d = o.case_inputs(fmt, H, L, D, 17 + H + L + S)
            ref = o.reference(d["kd"], d["vd"], d["q"], H, L, D)
            K, V = torch.from_numpy(d["kc"]).cuda(), torch.from_numpy(d["vc"]).cuda()
            sK = torch.from_numpy(d["ks"]).cuda().view(torch.float16)
            sV = torch.from_numpy(d["vs"]).cuda().view(torch.float16)
            q = torch.from_numpy(d["q"]).cuda().view(torch.float16)
            out = va.decode(fmt, K, V, sK, sV, q, H, L, D, S)
            torch.cuda.synchronize()
            err = np.abs(out.float().cpu().numpy() - ref)
            if not (err <= ATOL + RTOL * np.abs(ref)).all():
                print("FAIL", fmt, H, L, D, S, float(err.max()))
                fails += 1
    # grouped-query
    rng = np.random.default_rng(3)
    for fmt in ["q8+", "q4+", "q3+"]:
        for (B, Hq, Hkv, Lmax, D, S) in [(3, 8, 2, 300, 128, 3), (2, 8, 2, 200, 64, 2), (2, 16, 2, 150, 128, 1)]:
            lens = rng.integers(1, Lmax + 1, size=B).astype(np.int32)
            rows = B * Hkv * Lmax
            kx, vx, _ = o.gen_case(int(rng.integers(1 << 30)), 1, rows, D)
            qh = o.f2h(rng.standard_normal(B * Hq * D).astype(np.float32))
            bits = BITS[fmt]
            kc, ks = o.quantize(kx, 1, rows, D, bits)
            vc, vs = o.quantize(vx, 1, rows, D, bits)
            ref = o.reference_gqa(o.dequant(kc, ks, 1, rows, D, bits), o.dequant(vc, vs, 1, rows, D, bits),
                                  qh, lens, B, Hq, Hkv, Lmax, D)
            out = torch.empty(B * Hq * D, dtype=torch.float16, device="cuda")
            ws = torch.zeros(va.gqa_workspace_bytes(B, Hq, D, S), dtype=torch.uint8, device="cuda")
            b = va.DeviceBufs(torch.from_numpy(kc).cuda(), torch.from_numpy(vc).cuda(),
                              torch.from_numpy(ks).cuda().view(torch.float16),
                              torch.from_numpy(vs).cuda().view(torch.float16),
                              torch.from_numpy(qh).cuda().view(torch.float16), out, ws)
            va.decode_gqa(fmt, b, torch.from_numpy(lens).cuda(), B, Hq, Hkv, Lmax, D, S)
            torch.cuda.synchronize()
            err = np.abs(out.float().cpu().numpy() - ref)
            if not (err <= ATOL + RTOL * np.abs(ref)).all():
                print("FAIL gqa", fmt, B, Hq, Hkv, Lmax, D, S, float(err.max()))
                fails += 1
    if va.device_error() != 0:
        print("FAIL device error")
        fails += 1
    print("consumer", os.environ.get("VOLTATTN_CONSUMER"), "failures", fails)
    sys.exit(1 if fails else 0)


if __name__ == "__main__":
    main()
