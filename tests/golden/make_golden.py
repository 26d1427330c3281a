"""Generates the golden fixtures in this folder from the REFERENCE's own host code.

Run here (where the reference source exists) after `make -C oracle`:
    python tests/golden/make_golden.py

It loads oracle/_ref/libvoltattn_ref.so — the reference translation unit
src/voltattn.cu compiled unmodified from its own location — and records:

* selftest_ref.npz — for each selftest shape (src/voltattn.cu:913-916) and each
  data variant (f16-rounded, q8, q4, q3): the reference's `reference()` output
  (:770) on the exact values the reference attends over, plus the SHA-256 of
  the reference `quantize()` (:709) codes and scales of K and V.
* edge_quant.npz — an input with zero groups, tiny groups whose fp16 scale
  underflows, huge groups whose scale overflows, nan/inf elements and
  halfway values, with the reference's codes and scales for 8/4/3 bits.
* golden.json — SHA-256 digests: fp16 conversions over a fixed bit-pattern set
  (the reference's host __float2half / __half2float), and quantizer outputs of
  the larger configurations (selftest scale L=4096, the bench fill at
  L=16384, and the 1 %-outlier sweep input) used by the GPU quantizer tests.

Inputs are produced by the oracle's generators (std::mt19937 +
std::normal_distribution<float> in the reference's order, and the reference's
LCG fill), whose equality with the reference's own generator
(`fill_fast`, :960) is itself recorded here.
"""
from __future__ import annotations

import hashlib
import json
import os
import sys

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, os.path.join(HERE, "..", ".."))

from oracle.oracle import Oracle, RefLib, SELFTEST_CASES  # noqa: E402
from tests.golden.inputs import (HALF_PATTERN_STRIDE, edge_input, half_patterns,  # noqa: E402
                                 hash_config_inputs, HASH_CONFIGS)


def sha(*arrays) -> str:
    h = hashlib.sha256()
    for a in arrays:
        h.update(np.ascontiguousarray(a).tobytes())
    return h.hexdigest()


def main():
    o = Oracle()
    r = RefLib()
    out = {}
    gold = {}

    # fp16 conversions
    f = half_patterns()
    gold["f2h_stride"] = HALF_PATTERN_STRIDE
    gold["f2h_sha"] = sha(r.f2h(f))
    hall = np.arange(65536, dtype=np.uint32).astype(np.uint16)
    gold["h2f_sha"] = sha(r.h2f(hall))

    # selftest cases
    for (H, L, D, S) in SELFTEST_CASES:
        seed = o.selftest_seed(H, L, D, S)
        kx, vx, q = o.gen_case(seed, H, L, D)
        tag = f"H{H}_L{L}_D{D}_S{S}"
        out[f"{tag}_q"] = q
        kd = r.h2f(r.f2h(kx)); vd = r.h2f(r.f2h(vx))
        out[f"{tag}_f16_ref"] = r.reference(kd, vd, q, H, L, D)
        for bits in (8, 4, 3):
            kc, ks = r.quantize(kx, H, L, D, bits)
            vc, vs = r.quantize(vx, H, L, D, bits)
            gold[f"{tag}_q{bits}_sha"] = sha(kc, ks, vc, vs)
            kd = r.dequant(kc, ks, H, L, D, bits); vd = r.dequant(vc, vs, H, L, D, bits)
            out[f"{tag}_q{bits}_ref"] = r.reference(kd, vd, q, H, L, D)
            if (H, L, D) == (8, 129, 64):  # one case kept whole for readable diffs
                out[f"{tag}_q{bits}_kcodes"] = kc
                out[f"{tag}_q{bits}_kscales"] = ks
    np.savez_compressed(os.path.join(HERE, "selftest_ref.npz"), **out)

    # edge quantizer inputs
    H, L, D, x = edge_input()
    edge = {"x": x, "shape": np.array([H, L, D], np.int32)}
    for bits in (8, 4, 3):
        c, s = r.quantize(x, H, L, D, bits)
        edge[f"q{bits}_codes"] = c
        edge[f"q{bits}_scales"] = s
    np.savez_compressed(os.path.join(HERE, "edge_quant.npz"), **edge)

    # larger configurations: quantizer digests
    for name, cfg in HASH_CONFIGS.items():
        H, L, D = cfg["H"], cfg["L"], cfg["D"]
        kx, vx = hash_config_inputs(o, name)
        if cfg["gen"] == "fill_fast":  # the reference's own LCG, pinned here
            assert np.array_equal(kx, r.fill_fast(kx.size, cfg["kseed"]))
            assert np.array_equal(vx, r.fill_fast(vx.size, cfg["vseed"]))
        for bits in (8, 4, 3):
            kc, ks = r.quantize(kx, H, L, D, bits)
            vc, vs = r.quantize(vx, H, L, D, bits)
            gold[f"{name}_q{bits}_k_sha"] = sha(kc, ks)
            gold[f"{name}_q{bits}_v_sha"] = sha(vc, vs)
        print(name, "done", flush=True)

    with open(os.path.join(HERE, "golden.json"), "w") as fh:
        json.dump(gold, fh, indent=1, sort_keys=True)
    print("wrote", len(out), "arrays and", len(gold), "digests")


if __name__ == "__main__":
    main()
