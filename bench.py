#!/usr/bin/env python
"""Decode benchmark (the reference's `voltattn --bench`, src/voltattn.cu:967-1070,
re-derived for B200) with the driver's JSON contract.

A step is one batch-1 attention decode over all H=32 heads, D=128, L=16384
in format --fmt (default q4+), through the C ABI. The KV
cache is synthetic: fp32 N(0,1) K/V drawn on the GPU from a seeded generator
and packed by the GPU quantizer; q is fp16 N(0,1). Rank r of N decodes its own
sequence (weak scaling, no collective on the data path).

Timing: W warm-up steps plus a ~0.3 s soak, then exactly K steps replayed from
CUDA graphs, bracketed by barrier + synchronize; CUDA events on the launching
stream; max over ranks. Each step reads a different copy of the cache from a
rotation whose total exceeds 4x the L2 size, so L2 cannot serve the stream.

`--impl reference` times the reference's own CPU path (reference() of
src/voltattn.cu:769-794 over the dequantized cache, all host threads, built
from the reference source into oracle/_ref) on rank 0.
"""
from __future__ import annotations

import argparse
import json
import math
import os
import subprocess
import sys
import threading
import time

import numpy as np

ROOT = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, ROOT)

H, D = 32, 128
FORMAT_BITS = {"f16": 16, "f16+": 16, "q8": 8, "q8+": 8, "q4": 4, "q4+": 4, "q3+": 3, "bf16+": 16, "f8+": 8,
               "q4c+": 4}
# dram__bytes_read.sum + dram__bytes_write.sum per launch of the top kernel at
# L=16384, from one ncu capture per kernel taken at L=65536 (above the L2 size)
# and scaled to L=16384 by the rows processed (x 1/4): traffic grows in
# proportion to the rows, and the reads equal the algorithmic bytes there.
# Formats without a capture report None.
NCU_TRAFFIC_BYTES = {"q4+": int((285.290496e6 + 3.848704e6) / 4),
                     "q8+": int((553.788672e6 + 5.725184e6) / 4),
                     "f16+": int((1073.790e6 + 3.593472e6) / 4)}


def algorithmic_bytes(fmt: str, L: int) -> int:
    """K+V payload + fp16 group scales, q/out/workspace excluded
    (src/voltattn.cu:989-992)."""
    n = H * L * D
    bits = FORMAT_BITS[fmt]
    payload = 2 * n if bits == 16 else n if bits == 8 else n // 2 if bits == 4 else n * 3 // 8
    if fmt == "q4c+":  # K scales per (head, channel), V scales per row
        return 2 * payload + H * D * 2 + H * L * 2
    scales = 0 if bits == 16 else H * L * (D // 64) * 2
    return 2 * (payload + scales)


def parse_args():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=20000)
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--impl", choices=["ours", "reference"], default="ours")
    ap.add_argument("--fmt", default="q4+")
    ap.add_argument("--L", type=int, default=16384)
    ap.add_argument("--table", default="f16,f16+,q8,q8+,q4,q4+,q3+,bf16+,f8+,q4c+",
                    help="formats also timed for the per-format table (empty: none)")
    ap.add_argument("--no-cpu", action="store_true", help="skip the cpu_baseline leg")
    ap.add_argument("--no-extra", action="store_true", help="skip the GQA / split-L extra measurements")
    ap.add_argument("--no-sweep", action="store_true", help="skip the context-length sweep (config 4)")
    ap.add_argument("--profile", action="store_true",
                    help="profiling driver for ncu: W+K plain launches of --fmt at --L (one cache, no graphs)")
    ap.add_argument("--prefill-lq", type=int, default=0,
                    help="with --profile: prefill of this many tokens (cache of --L rows, 32/8 heads) instead")
    ap.add_argument("--timeline", action="store_true",
                    help="per-CTA event timeline of the tile kernel (needs `make timeline`)")
    ap.add_argument("--gqa-batch", type=int, default=0,
                    help="with --profile: the batched GQA decode of config 5 with this many sequences instead")
    return ap.parse_args()


# ---------------------------------------------------------------- helpers ----

def measured_peaks():
    try:
        with open(os.path.join(ROOT, "MEASURED_PEAKS.json")) as fh:
            return json.load(fh), "measured"
    except OSError:
        return {"hbm_gbs": 6650.0, "bf16_tflops": 1590.0}, "fallback"


class ClockSampler:
    """nvidia-smi clocks / throttle reasons sampled every 50 ms."""

    def __init__(self, uuid: str | None):
        self.uuid = uuid
        self.proc = None
        self.lines = []

    def __enter__(self):
        cmd = ["nvidia-smi", "--query-gpu=clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
               "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
               "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap",
               "--format=csv,noheader,nounits", "-lms", "50"]
        if self.uuid:
            cmd += ["-i", self.uuid]
        try:
            self.proc = subprocess.Popen(cmd, stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
            self.th = threading.Thread(target=self._read, daemon=True)
            self.th.start()
        except OSError:
            self.proc = None
        return self

    def _read(self):
        for line in self.proc.stdout:
            self.lines.append(line.strip())

    def __exit__(self, *a):
        if self.proc:
            self.proc.terminate()
            try:
                self.proc.wait(timeout=5)
            except subprocess.TimeoutExpired:
                self.proc.kill()
            self.th.join(timeout=2)

    def summary(self):
        sm, mx, reasons = [], None, set()
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        for ln in self.lines:
            f = [x.strip() for x in ln.split(",")]
            if len(f) < 8:
                continue
            try:
                sm.append(float(f[0]))
                mx = float(f[1])
            except ValueError:
                continue
            for n, v in zip(names, f[4:8]):
                if v.lower() == "active":
                    reasons.add(n)
        return {"sm_mhz": float(np.median(sm)) if sm else None, "sm_max_mhz": mx, "reasons": sorted(reasons),
                "samples": len(sm)}


def cpu_sample_plan(t_full: float, K: int, budget_s: float):
    """Fraction of the full decode one CPU step covers so that K steps take
    about budget_s: whole heads while that is enough, else a prefix of the
    positions of one head."""
    frac = min(1.0, budget_s / max(1e-9, K * t_full))
    heads = max(1, min(H, int(math.floor(frac * H))))
    if frac * H >= 1.0:
        return heads, None
    return 1, max(64, int(frac * H * 1.0 * 16384))


# ------------------------------------------------------------ CPU paths -------

def cpu_reference_setup(L: int, fmt: str, seed: int = 1234):
    """The reference's CPU decode inputs: exactly dequantized K/V (fp32) and
    fp16 q, quantized by the reference's own quantize() where built."""
    from oracle.oracle import REF_SO, Oracle, RefLib
    o = Oracle()
    kind = "reference" if os.path.exists(REF_SO) else "port"
    lib = RefLib() if kind == "reference" else o
    rng = np.random.default_rng(seed)
    kx = rng.standard_normal(H * L * D, dtype=np.float32)
    vx = rng.standard_normal(H * L * D, dtype=np.float32)
    q = o.f2h(rng.standard_normal(H * D, dtype=np.float32))
    bits = FORMAT_BITS[fmt]
    if bits == 16:
        kd, vd = o.round_to_half(kx), o.round_to_half(vx)
    else:
        kc, ks = lib.quantize(kx, H, L, D, bits)
        vc, vs = lib.quantize(vx, H, L, D, bits)
        kd, vd = lib.dequant(kc, ks, H, L, D, bits), lib.dequant(vc, vs, H, L, D, bits)
    return lib, kind, kd, vd, q


def cpu_time_step(lib, kd, vd, q, L, heads, positions, threads):
    if positions is None:
        n = heads * L * D
        t = time.perf_counter()
        lib.reference(kd[:n], vd[:n], q[:heads * D], heads, L, D, threads=threads)
        return time.perf_counter() - t, heads / H
    kh = np.ascontiguousarray(kd[:L * D].reshape(L, D)[:positions])
    vh = np.ascontiguousarray(vd[:L * D].reshape(L, D)[:positions])
    t = time.perf_counter()
    lib.reference(kh, vh, q[:D], 1, positions, D, threads=1)
    return time.perf_counter() - t, positions / (H * L)


def cpu_baseline_leg(L, fmt):
    threads = os.cpu_count() or 1
    lib, kind, kd, vd, q = cpu_reference_setup(L, fmt)
    t_full, _ = cpu_time_step(lib, kd, vd, q, L, H, None, threads)
    runs = max(1, min(200, int(10.0 / max(t_full, 1e-6))))
    t0 = time.perf_counter()
    for _ in range(runs):
        cpu_time_step(lib, kd, vd, q, L, H, None, threads)
    dt = time.perf_counter() - t0
    return {"value": runs / dt, "unit": "tok/s", "cores": threads, "kind": kind,
            "sample": f"{runs} full decodes (H={H}, D={D}, L={L}, {fmt} cache dequantized to fp32 by the "
                      f"reference's dq), heads over {threads} threads, double-precision reference()"}


REF_FMT_INDEX = {"f16": 0, "f16+": 1, "q8": 2, "q8+": 3, "q4": 4, "q4+": 5, "q3+": 6}


def reference_kernels_leg(L=16384, n=200):
    """The reference's own kernels rebuilt for sm_100a (oracle/_ref, its
    unmodified translation unit) on this GPU: n back-to-back launch() calls
    per format (its decode kernel plus its combine, legacy default stream,
    CUDA events around the loop), the reference bench's split rule
    (src/voltattn.cu:1026), caches quantized by the reference's own host
    quantize() and rotated over > 4x L2. The GPU speed bar for our kernels."""
    import torch
    from oracle.oracle import RefLib
    lib = RefLib()
    dev = torch.device("cuda", 0)
    rng = np.random.default_rng(99)
    n_el = H * L * D
    kx = rng.standard_normal(n_el, dtype=np.float32)
    vx = rng.standard_normal(n_el, dtype=np.float32)
    q = torch.from_numpy(lib.f2h(rng.standard_normal(H * D, dtype=np.float32)).view(np.int16)).to(dev)
    nsm = torch.cuda.get_device_properties(dev).multi_processor_count
    S = max(1, min(nsm * 2 // H, (L + 511) // 512))
    out = torch.empty(H * D, dtype=torch.int16, device=dev)
    ws = torch.empty(H * S * (D + 2), dtype=torch.float32, device=dev)
    l2 = getattr(torch.cuda.get_device_properties(dev), "L2_cache_size", 126 << 20)
    res = {}
    packed = {}
    for f, idx in REF_FMT_INDEX.items():
        bits = FORMAT_BITS[f]
        if bits == 16:
            tensors = [torch.from_numpy(lib.f2h(x).view(np.int16)).to(dev) for x in (kx, vx)] + [None, None]
        else:
            if bits not in packed:
                kc, ks = lib.quantize(kx, H, L, D, bits)
                vc, vs = lib.quantize(vx, H, L, D, bits)
                packed[bits] = [torch.from_numpy(a.view(np.uint8)).to(dev) for a in (kc, vc, ks, vs)]
            tensors = packed[bits]
        nbytes = algorithmic_bytes(f, L)
        copies = max(2, math.ceil(4 * l2 / nbytes))
        caches = [tensors] + [[None if t is None else t.clone() for t in tensors] for _ in range(copies - 1)]
        ptrs = [tuple(None if t is None else t.data_ptr() for t in c) for c in caches]
        torch.cuda.synchronize(dev)
        ms = lib.time_launches(idx, ptrs, q.data_ptr(), out.data_ptr(), ws.data_ptr(), H, L, D, S, n)
        res[f] = {"ms": ms, "gbs": nbytes / (ms * 1e6), "tok_s": 1e3 / ms, "splits": S}
        del caches
        torch.cuda.empty_cache()
    return {"workload": f"the reference's launch() rebuilt for sm_100a, batch-1 decode H={H} D={D} L={L}",
            "timing": f"{n} back-to-back launches per format, CUDA events, caches rotated over > 4x L2",
            "formats": res}


def run_reference_arm(args, rank):
    if rank != 0:
        return
    L, fmt = args.L, args.fmt
    threads = os.cpu_count() or 1
    lib, kind, kd, vd, q = cpu_reference_setup(L, fmt)
    t_full, _ = cpu_time_step(lib, kd, vd, q, L, H, None, threads)
    heads, positions = cpu_sample_plan(t_full, args.steps + args.warmup, 120.0)
    for _ in range(args.warmup):
        cpu_time_step(lib, kd, vd, q, L, heads, positions, threads)
    total, covered = 0.0, 0.0
    for _ in range(args.steps):
        dt, frac = cpu_time_step(lib, kd, vd, q, L, heads, positions, threads)
        total += dt
        covered += frac
    value = covered / total  # full decodes per second
    sample = (f"each step: {heads} of {H} heads, all {L} positions" if positions is None else
              f"each step: 1 head, first {positions} of {L} positions") + \
        f"; {fmt} cache dequantized by the reference's dq; reference() on {threads if positions is None else 1} threads"
    line = {"impl": "reference", "metric": f"decode tok/s (batch 1, H={H}, D={D}, L={L}, {fmt})",
            "value": value, "unit": "tok/s", "n_gpus": args.gpus, "steps": args.steps, "warmup": args.warmup,
            "ms_per_step": 1e3 / value, "higher_is_better": True, "scaling": "weak", "vs_baseline": None,
            "dtype": "f64", "data": "synthetic: fp32 N(0,1) K/V, fp16 N(0,1) q, seeded",
            "config": {"workload": f"batch-1 decode H={H} D={D} L={L} fmt={fmt}", "H": H, "D": D, "L": L,
                       "fmt": fmt},
            "cpu_baseline": {"value": value, "unit": "tok/s", "cores": threads if positions is None else 1,
                             "kind": kind, "sample": sample},
            "e2e": {"value": value, "unit": "tok/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}}
    if kind == "reference" and not args.no_extra:
        try:
            import torch
            if torch.cuda.is_available():
                line["extra"] = {"reference_kernels_sm100a": reference_kernels_leg(L)}
        except Exception as e:  # the CPU line stands without the GPU speed bar
            line["extra"] = {"reference_kernels_sm100a": {"unavailable": f"{type(e).__name__}: {e}"}}
    print(json.dumps(line), flush=True)


# ------------------------------------------------------------ GPU path --------

def make_cache(va, torch, fmt, L, seed, dev, outliers=False):
    """Synthetic cache of one sequence: fp32 N(0,1) K/V from a seeded GPU
    generator, packed into fmt by the GPU quantizers. outliers: 1 % of the K
    entries (a seeded mask) scaled x8, which stresses the group scales
    (BASELINE config 4)."""
    g = torch.Generator(device=dev)
    g.manual_seed(seed)
    n = H * L * D
    kx = torch.randn(n, generator=g, device=dev, dtype=torch.float32)
    vx = torch.randn(n, generator=g, device=dev, dtype=torch.float32)
    if outliers:
        kx[torch.rand(n, generator=g, device=dev) < 0.01] *= 8.0
    bits = FORMAT_BITS[fmt]
    if fmt == "bf16+":
        K, V, sK, sV = kx.bfloat16(), vx.bfloat16(), None, None
    elif fmt == "f8+":
        K, sK = va.quantize_f8(kx, H, L, D)
        V, sV = va.quantize_f8(vx, H, L, D)
    elif fmt == "q4c+":
        K, sK = va.quantize_kchan(kx, 4, H, L, D)
        V, sV = va.quantize_vtok(vx, 4, H, L, D)
    elif bits == 16:
        K, V, sK, sV = kx.half(), vx.half(), None, None
    else:
        K, sK = va.quantize(kx, bits, H, L, D)
        V, sV = va.quantize(vx, bits, H, L, D)
    del kx, vx
    return K, V, sK, sV


def time_format(va, torch, fmt, L, K_steps, W, dev, dist, seed, soak_s=0.3, splits=None, outliers=False):
    """Returns (ms_per_step, S, copies, launches_per_step) for K_steps decodes."""
    nbytes = algorithmic_bytes(fmt, L)
    l2 = getattr(torch.cuda.get_device_properties(dev), "L2_cache_size", 126 << 20)
    copies = max(2, math.ceil(4 * l2 / nbytes))
    base = make_cache(va, torch, fmt, L, seed, dev, outliers)
    caches = [base] + [tuple(None if t is None else t.clone() for t in base) for _ in range(copies - 1)]
    q = torch.randn(H * D, device=dev, generator=torch.Generator(device=dev).manual_seed(seed + 1)).half()
    out = torch.empty(H * D, dtype=torch.float16, device=dev)
    S = splits or va.suggest_splits(fmt, H, L, D)
    ws = va.new_workspace(H, D, S, dev)
    bufs = [va.DeviceBufs(*c, q, out, ws) for c in caches]
    stream = torch.cuda.Stream(device=dev)

    def step(i):
        va.launch(fmt, bufs[i % copies], H, L, D, S, stream)

    # the caches and the zeroed workspace come from the default stream: make
    # them complete before the decode stream reads them
    torch.cuda.synchronize(dev)
    with torch.cuda.stream(stream):
        for i in range(max(3, W)):
            step(i)
    torch.cuda.synchronize(dev)
    chunk = min(K_steps, 32 * copies)
    graphs = []

    def capture(n):
        gph = torch.cuda.CUDAGraph()
        with torch.cuda.graph(gph, stream=stream):
            for i in range(n):
                step(i)
        return gph

    main = capture(chunk)
    reps, tail = divmod(K_steps, chunk)
    tail_g = capture(tail) if tail else None
    torch.cuda.synchronize(dev)
    # soak (untimed): same work, lets clocks settle for the sampler
    t_end = time.perf_counter() + soak_s
    while time.perf_counter() < t_end:
        main.replay()
        torch.cuda.synchronize(dev)
    e0 = torch.cuda.Event(enable_timing=True)
    e1 = torch.cuda.Event(enable_timing=True)
    if dist:
        dist.barrier()
    torch.cuda.synchronize(dev)
    e0.record(stream)
    with torch.cuda.stream(stream):
        for _ in range(reps):
            main.replay()
        if tail_g is not None:
            tail_g.replay()
    e1.record(stream)
    torch.cuda.synchronize(dev)
    if dist:
        dist.barrier()
    ms = e0.elapsed_time(e1)
    if dist:
        t = torch.tensor([ms], device=dev, dtype=torch.float64)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        ms = float(t.item())
    launches = 1 if fmt.endswith("+") else 2
    del graphs
    return ms / K_steps, S, copies, launches


def e2e_leg(va, torch, fmt, L, K_steps, dev, dist, seed):
    """End to end through the public API, as a serving loop runs it: per step
    the host writes this step's q into pinned memory and calls va_decode_host
    (H2D of q, the decode storing its fp16 output into pinned memory; a cached
    CUDA graph per cache copy; returns synchronized), then reads the output.
    Caches rotate over > 4x L2 so every decode reads HBM."""
    import math
    nbytes = algorithmic_bytes(fmt, L)
    l2 = getattr(torch.cuda.get_device_properties(dev), "L2_cache_size", 126 << 20)
    copies = max(2, math.ceil(4 * l2 / nbytes))
    base = make_cache(va, torch, fmt, L, seed, dev)
    caches = [base] + [tuple(None if t is None else t.clone() for t in base) for _ in range(copies - 1)]
    S = va.suggest_splits(fmt, H, L, D)
    ws = va.new_workspace(H, D, S, dev)
    nq = 64
    q_src = torch.randn(nq, H * D).half()
    q_pin = torch.empty(H * D, dtype=torch.float16).pin_memory()
    out_pin = torch.empty(H * D, dtype=torch.float16).pin_memory()
    out_sink = torch.empty(nq, H * D, dtype=torch.float16)
    q = torch.empty(H * D, dtype=torch.float16, device=dev)
    out = torch.empty(H * D, dtype=torch.float16, device=dev)
    stream = torch.cuda.Stream(device=dev)
    bufs = [va.DeviceBufs(*c, q, out, ws) for c in caches]
    torch.cuda.synchronize(dev)  # inputs made on the default stream are complete

    # host side through numpy views of the pinned buffers (cheaper than torch ops)
    q_src_np, q_pin_np = q_src.numpy(), q_pin.numpy()
    out_pin_np, out_sink_np = out_pin.numpy(), out_sink.numpy()
    steps = min(K_steps, 20000)

    # va_decode_host per cache copy with its arguments bound once (va.HostStep):
    # q from pinned memory, decode, output to pinned memory, synchronized; a
    # cached CUDA graph after the first call
    host_steps = [va.HostStep(fmt, bb, q_pin, out_pin, H, L, D, S, stream) for bb in bufs]

    def one(i):
        q_pin_np[:] = q_src_np[i % nq]
        host_steps[i % copies]()
        out_sink_np[i % nq] = out_pin_np

    for i in range(2 * copies):  # every copy's first call captures its graph
        one(i)
    if dist:
        dist.barrier()
    t0 = time.perf_counter()
    for i in range(steps):
        one(i)
    dt = time.perf_counter() - t0
    if dist:
        t = torch.tensor([dt], device=dev, dtype=torch.float64)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        dt = float(t.item())
    n = dist.get_world_size() if dist else 1
    return {"value": n * steps / dt, "unit": "tok/s", "h2d_bytes_per_step": H * D * 2,
            "d2h_bytes_per_step": H * D * 2, "steps": steps,
            "note": "KV cache resident in HBM (decode state), rotating over > 4x L2; per step: q written to "
                    "pinned memory, va_decode_host (H2D q by va_copy_small from device-mapped pinned memory, decode "
                    "storing its output into pinned memory, as one cached CUDA graph; returns synchronized), "
                    "output read"}


def make_gqa(va, torch, dev, seed, fmt, B, Hq, Hkv, Lmax, S):
    """Synthetic batched grouped-query state: per-sequence lengths uniform in
    [1024, Lmax] from a seed, K/V drawn on the GPU and packed by the GPU
    quantizer into a capacity-padded [B][Hkv][Lmax] cache, fp16 q."""
    g = torch.Generator(device="cpu").manual_seed(seed)
    lens = torch.randint(1024, Lmax + 1, (B,), generator=g, dtype=torch.int32)
    rows = B * Hkv * Lmax
    gd = torch.Generator(device=dev).manual_seed(seed)
    bits = FORMAT_BITS[fmt]
    parts = []
    for _ in range(2):  # K then V, quantized in slices to bound the fp32 staging
        codes = torch.empty(rows * D * bits // 8, dtype=torch.uint8, device=dev)
        scales = torch.empty(rows * (D // 64), dtype=torch.float16, device=dev)
        step_rows = 1 << 20
        for r0 in range(0, rows, step_rows):
            r1 = min(rows, r0 + step_rows)
            x = torch.randn((r1 - r0) * D, generator=gd, device=dev)
            va.quantize(x, bits, 1, r1 - r0, D, codes[r0 * D * bits // 8: r1 * D * bits // 8],
                        scales[r0 * (D // 64): r1 * (D // 64)])
        parts.append((codes, scales))
    (K, sK), (V, sV) = parts
    q = torch.randn(B * Hq * D, generator=gd, device=dev).half()
    out = torch.empty(B * Hq * D, dtype=torch.float16, device=dev)
    ws = torch.zeros(va.gqa_workspace_bytes(B, Hq, D, S), dtype=torch.uint8, device=dev)
    nbytes = int(lens.sum()) * Hkv * 2 * (D * bits // 8 + 2 * (D // 64))
    return va.DeviceBufs(K, V, sK, sV, q, out, ws), lens.to(dev), nbytes


def paged_from(torch, dev, b, lens_d, B, Hkv, Lmax, fmt, page_rows, seed):
    """The same cache scattered into a pool of pages in a seeded random order:
    K/V [num_pages][Hkv][page_rows] rows, scales alike, block table [B][max_pages]."""
    bits = FORMAT_BITS[fmt]
    rb, ng = D * bits // 8, D // 64
    max_pages = (Lmax + page_rows - 1) // page_rows
    num_pages = B * max_pages
    g = torch.Generator(device="cpu").manual_seed(seed)
    perm = torch.randperm(num_pages, generator=g).to(dev)

    def scatter(t, width):
        src = t.view(B, Hkv, max_pages, page_rows, width).permute(0, 2, 1, 3, 4).reshape(num_pages, Hkv, page_rows,
                                                                                           width)
        pool = torch.empty_like(src)
        pool.index_copy_(0, perm, src)
        return pool.reshape(-1)

    pK, pV = scatter(b.K, rb), scatter(b.V, rb)
    psK = scatter(b.scK.view(torch.uint8), 2 * ng).view(torch.float16)
    psV = scatter(b.scV.view(torch.uint8), 2 * ng).view(torch.float16)
    table = perm.view(B, max_pages).to(torch.int32)
    return pK, pV, psK, psV, table, max_pages, num_pages


def paged_leg(va, torch, dev, steps, page_rows=256, seed=4242, fmt="q4+", B=64, Hq=32, Hkv=8, Lmax=32768, S=4):
    """Config 5 over a paged cache: the same sequences and lengths, the cache in
    pages of `page_rows` rows at shuffled pool positions (va_decode_paged)."""
    b, lens_d, nbytes = make_gqa(va, torch, dev, seed, fmt, B, Hq, Hkv, Lmax, S)
    pK, pV, psK, psV, table, max_pages, num_pages = paged_from(torch, dev, b, lens_d, B, Hkv, Lmax, fmt, page_rows,
                                                              seed)
    pb = va.DeviceBufs(pK, pV, psK, psV, b.q, b.out, b.ws)
    b.K = b.V = b.scK = b.scV = None  # the contiguous cache is no longer needed
    stream = torch.cuda.Stream(device=dev)
    torch.cuda.synchronize(dev)  # inputs made on the default stream are complete

    def run():
        va.decode_paged(fmt, pb, table, max_pages, lens_d, B, Hq, Hkv, page_rows, num_pages, D, S, stream)

    with torch.cuda.stream(stream):
        for _ in range(3):
            run()
    torch.cuda.synchronize(dev)
    n = max(3, min(steps, 200))
    gph = torch.cuda.CUDAGraph()
    with torch.cuda.graph(gph, stream=stream):
        for _ in range(n):
            run()
    e0 = torch.cuda.Event(enable_timing=True)
    e1 = torch.cuda.Event(enable_timing=True)
    with torch.cuda.stream(stream):
        gph.replay()
        e0.record(stream)
        gph.replay()
        e1.record(stream)
    torch.cuda.synchronize(dev)
    ms = e0.elapsed_time(e1) / n
    return {"workload": f"paged GQA decode B={B} Hq={Hq} Hkv={Hkv} D={D} lens~U[1024,{Lmax}] {fmt}, "
                        f"pages of {page_rows} rows in shuffled order",
            "ms": ms, "tok_s": B * 1e3 / ms, "gbs": nbytes / (ms * 1e6), "bytes": nbytes, "splits": S,
            "page_rows": page_rows, "steps": n, "launches_per_step": 1}


def gqa_leg(va, torch, dev, steps, seed=4242, fmt="q4+", B=64, Hq=32, Hkv=8, Lmax=32768, S=4):
    """batched grouped-query decode, 64 sequences, 32 query
    heads over 8 KV heads, per-sequence length uniform in [1024, 32768] from a
    seed, INT4 cache. tok/s = B tokens per step. S = 4 splits per KV stream
    (2048 units over the grid) measured best for the grouped-query tile
    kernel (S = 1, 2, 4, 8, 16: 0.354, 0.280, 0.247, 0.256, 0.291 ms)."""
    b, lens_d, nbytes = make_gqa(va, torch, dev, seed, fmt, B, Hq, Hkv, Lmax, S)
    stream = torch.cuda.Stream(device=dev)
    torch.cuda.synchronize(dev)  # inputs made on the default stream are complete
    with torch.cuda.stream(stream):
        for _ in range(3):
            va.decode_gqa(fmt, b, lens_d, B, Hq, Hkv, Lmax, D, S, stream)
    torch.cuda.synchronize(dev)
    n = max(3, min(steps, 200))
    gph = torch.cuda.CUDAGraph()
    with torch.cuda.graph(gph, stream=stream):
        for _ in range(n):
            va.decode_gqa(fmt, b, lens_d, B, Hq, Hkv, Lmax, D, S, stream)
    e0 = torch.cuda.Event(enable_timing=True)
    e1 = torch.cuda.Event(enable_timing=True)
    with torch.cuda.stream(stream):
        gph.replay()
        e0.record(stream)
        gph.replay()
        e1.record(stream)
    torch.cuda.synchronize(dev)
    ms = e0.elapsed_time(e1) / n
    return {"workload": f"batched GQA decode B={B} Hq={Hq} Hkv={Hkv} D={D} lens~U[1024,{Lmax}] {fmt}",
            "ms": ms, "tok_s": B * 1e3 / ms, "gbs": nbytes / (ms * 1e6), "bytes": nbytes, "splits": S,
            "steps": n, "launches_per_step": 1}


def gqa_sharded_leg(va, torch, dev, dist, world, rank, steps, seed=4242, fmt="q4+", B=64, Hq=32, Hkv=8, Lmax=32768,
                    S=4):
    """BASELINE config 5 sharded by sequence over the ranks (BatchSharding:
    rank r decodes sequences [b0, b1) of the same seeded batch, no collective
    on the data path). Each rank times a CUDA graph of back-to-back decodes of
    its shard; tok/s = B / (max over ranks of the per-step time)."""
    from voltattn_b200.launcher import split_range
    g = torch.Generator(device="cpu").manual_seed(seed)
    lens_all = torch.randint(1024, Lmax + 1, (B,), generator=g, dtype=torch.int32)
    b0, b1 = split_range(B, world, rank, align=1)
    Bl = b1 - b0
    b, lens_d, nbytes = make_gqa(va, torch, dev, seed + 1 + rank, fmt, Bl, Hq, Hkv, Lmax, S)
    lens_d = lens_all[b0:b1].to(dev)
    nbytes = int(lens_all[b0:b1].sum()) * Hkv * 2 * (D * FORMAT_BITS[fmt] // 8 + 2 * (D // 64))
    stream = torch.cuda.Stream(device=dev)
    torch.cuda.synchronize(dev)
    with torch.cuda.stream(stream):
        for _ in range(3):
            va.decode_gqa(fmt, b, lens_d, Bl, Hq, Hkv, Lmax, D, S, stream)
    torch.cuda.synchronize(dev)
    n = max(3, min(steps, 200))
    gph = torch.cuda.CUDAGraph()
    with torch.cuda.graph(gph, stream=stream):
        for _ in range(n):
            va.decode_gqa(fmt, b, lens_d, Bl, Hq, Hkv, Lmax, D, S, stream)
    torch.cuda.synchronize(dev)
    dist.barrier()
    e0 = torch.cuda.Event(enable_timing=True)
    e1 = torch.cuda.Event(enable_timing=True)
    with torch.cuda.stream(stream):
        e0.record(stream)
        gph.replay()
        e1.record(stream)
    torch.cuda.synchronize(dev)
    t = torch.tensor([e0.elapsed_time(e1) / n, float(nbytes)], device=dev, dtype=torch.float64)
    tmax = t[:1].clone()
    dist.all_reduce(tmax, op=dist.ReduceOp.MAX)
    tb = t[1:].clone()
    dist.all_reduce(tb, op=dist.ReduceOp.SUM)
    ms = float(tmax.item())
    return {"workload": f"batched GQA decode B={B} Hq={Hq} Hkv={Hkv} D={D} lens~U[1024,{Lmax}] {fmt}, "
                        f"sequences sharded over {world} GPUs", "ms": ms, "tok_s": B * 1e3 / ms,
            "gbs_total": float(tb.item()) / (ms * 1e6), "splits": S, "steps": n, "scaling": "strong",
            "launches_per_step_per_rank": 1}


def make_prefill(va, torch, dev, fmt, Hq, Hkv, L, Lq, seed):
    """One sequence's cache of L rows per KV head (its last Lq rows are the new
    tokens) in format fmt, quantized on the GPU, and the tokens' fp16 queries."""
    g = torch.Generator(device=dev).manual_seed(seed)
    rows = Hkv * L
    bits = FORMAT_BITS[fmt]
    kx = torch.randn(rows * D, device=dev, generator=g)
    vx = torch.randn(rows * D, device=dev, generator=g)
    if bits == 16:
        K, V, sK, sV = kx.half(), vx.half(), None, None
    else:
        K, sK = va.quantize(kx, bits, 1, rows, D)
        V, sV = va.quantize(vx, bits, 1, rows, D)
    del kx, vx
    q = torch.randn(Hq * Lq * D, device=dev, generator=g).half()
    out = torch.empty_like(q)
    return va.DeviceBufs(K, V, sK, sV, q, out)


def prefill_flops(Hq, L, Lq):
    """Algorithmic FLOPs of a causal prefill: 2 D multiply-adds (QK and PV) per
    visible (token, row) pair, token i seeing L - Lq + 1 + i rows."""
    pairs = Lq * (L - Lq) + Lq * (Lq + 1) // 2
    return 4.0 * D * Hq * pairs


def prefill_leg(va, torch, dev, fmt="q4+", Hq=32, Hkv=8, L=8192, Lq=8192, reps=10, staged=True):
    """Prompt prefill on the tcgen05 kernel: Lq tokens over a cache of L rows
    (L = Lq: a fresh prompt), 32 query / 8 KV heads. TFLOP/s of the causal
    work (no flops counted for masked pairs), against the measured bf16 dense
    peak (the kernel computes fp16 x fp16 -> fp32). staged: the cache is
    converted once to fp16 in a workspace and the tiles move by tensor copies
    (the conversion pass is inside the timed launches); unstaged: every CTA
    converts the blocks it reads."""
    b = make_prefill(va, torch, dev, fmt, Hq, Hkv, L, Lq, 5150)
    if staged:
        b.ws = torch.empty(va.prefill_workspace_bytes(Hkv, L, D), dtype=torch.uint8, device=dev)
    stream = torch.cuda.Stream(device=dev)
    torch.cuda.synchronize(dev)  # inputs made on the default stream are complete
    with torch.cuda.stream(stream):
        for _ in range(3):
            va.prefill(fmt, b, Hq, Hkv, L, Lq, D, stream, staged=staged)
    torch.cuda.synchronize(dev)
    e0 = torch.cuda.Event(enable_timing=True)
    e1 = torch.cuda.Event(enable_timing=True)
    with torch.cuda.stream(stream):
        e0.record(stream)
        for _ in range(reps):
            va.prefill(fmt, b, Hq, Hkv, L, Lq, D, stream, staged=staged)
        e1.record(stream)
    torch.cuda.synchronize(dev)
    ms = e0.elapsed_time(e1) / reps
    flops = prefill_flops(Hq, L, Lq)
    peaks, kind = measured_peaks()
    tf = flops / (ms * 1e9)
    err = va.device_error()
    return {"workload": f"prefill Hq={Hq} Hkv={Hkv} D={D} L={L} Lq={Lq} causal {fmt}"
                        + ("" if staged else ", unstaged (per-CTA conversion)"), "ms": ms,
            "tok_s": Lq * 1e3 / ms, "tflops": tf, "flops": flops,
            "roofline": {"bound": "tensor", "achieved": tf, "peak": peaks["bf16_tflops"], "unit": "TFLOP/s",
                         "frac": tf / peaks["bf16_tflops"], "peak_kind": f"{kind} (cuBLAS bf16 burst)"},
            "reps": reps, "device_error": err}


SWEEP_FORMATS = ("f16", "f16+", "q8", "q8+", "q4", "q4+", "q3+")
SWEEP_L = (1024, 4096, 16384, 65536)


def sweep_leg(va, torch, dev, probe, steps=300):
    """batch-1 decode, H=32, D=128, every reference format
    at L in {1024, 4096, 16384, 65536}, N(0,1) q/K/V with 1 % of the K entries
    scaled x8; MBU against the live read probe per (format, L). Each point is
    a CUDA graph of back-to-back decodes over rotating copies (> 4x L2)."""
    out = {}
    for L in SWEEP_L:
        row = {}
        for f in SWEEP_FORMATS:
            ms, S, _, _ = time_format(va, torch, f, L, steps, 3, dev, None, 4000 + L, soak_s=0.0, outliers=True)
            gbs = algorithmic_bytes(f, L) / (ms * 1e6)
            row[f] = {"us": round(ms * 1e3, 3), "gbs": round(gbs, 1), "mbu_probe": round(gbs / probe, 4),
                      "tok_s": round(1e3 / ms, 1), "splits": S}
            torch.cuda.empty_cache()
        out[str(L)] = row
    return {"workload": f"batch-1 decode H={H} D={D}, 1% of K x8, formats {','.join(SWEEP_FORMATS)}",
            "probe_gbs": probe, "points": out}


def accuracy_leg(va, torch, dev, L=4096, seed=31):
    """H=32, D=128, L=4096, q/K/V N(0,1); the quantized
    decodes against the fp16 attention output (f16+ over the fp16-rounded
    cache), i.e. the quantization error the reference's selftest keeps out of
    its gate. Max and mean |difference| over the H*D outputs."""
    g = torch.Generator(device=dev).manual_seed(seed)
    n = H * L * D
    kx = torch.randn(n, generator=g, device=dev)
    vx = torch.randn(n, generator=g, device=dev)
    q = torch.randn(H * D, generator=g, device=dev).half()
    ref = va.decode("f16+", kx.half(), vx.half(), None, None, q, H, L, D, va.suggest_splits("f16+", H, L, D)).float()
    res = {"workload": f"H={H} D={D} L={L}, N(0,1) q/K/V, vs the fp16 (f16+) attention output",
           "ref_abs_mean": float(ref.abs().mean())}
    for f in ("q8+", "q4+", "q3+"):
        bits = FORMAT_BITS[f]
        K, sK = va.quantize(kx, bits, H, L, D)
        V, sV = va.quantize(vx, bits, H, L, D)
        got = va.decode(f, K, V, sK, sV, q, H, L, D, va.suggest_splits(f, H, L, D)).float()
        err = (got - ref).abs()
        res[f] = {"max_abs": float(err.max()), "mean_abs": float(err.mean())}
    return res


def splitl_leg(va, torch, dev, dist, world, steps, fmt="q4+", L=131072, S=None):
    """BASELINE config 3 across GPUs: one sequence of L positions split into
    contiguous ranges per rank; each rank decodes its range into per-head
    partials, which are exchanged and merged (strong scaling: total work
    fixed). Two exchanges are timed: NCCL all-gather + combine kernel, and the
    fused peer-memory exchange-and-combine kernel over NVLink."""
    from voltattn_b200.launcher import SplitL, SplitLPeer
    sl = SplitLPeer(L, H, D, dev)
    Lr = sl.local_len
    # one seeded cache of the whole sequence (the same on every rank); rank r
    # keeps its contiguous range [j0, j1) of every head's rows
    full = make_cache(va, torch, fmt, L, 777, dev)
    rb = D * FORMAT_BITS[fmt] // 8

    def rows(t, width):
        return None if t is None else t.view(H, L, width)[:, sl.j0:sl.j1].contiguous().view(-1)

    K, V = rows(full[0], rb), rows(full[1], rb)
    sK = rows(full[2].view(torch.uint8), 2 * (D // 64)).view(torch.float16)
    sV = rows(full[3].view(torch.uint8), 2 * (D // 64)).view(torch.float16)
    q = torch.randn(H * D, device=dev, generator=torch.Generator(device=dev).manual_seed(5)).half()
    S = S or va.suggest_splits(fmt, H, Lr, D)
    ws = va.new_workspace(H, D, S, dev)
    out_local = torch.empty(H * D, dtype=torch.float16, device=dev)
    out = torch.empty(H * D, dtype=torch.float16, device=dev)
    partial = torch.empty(H, D + 2, dtype=torch.float32, device=dev)
    b = va.DeviceBufs(K, V, sK, sV, q, out_local, ws)

    def pfn(j0, j1):
        va.decode_partial(fmt, b, H, Lr, D, S, partial)
        return partial

    def timed(step):
        for _ in range(5):
            step()
        torch.cuda.synchronize(dev)
        n = max(5, min(steps, 500))
        dist.barrier()
        e0 = torch.cuda.Event(enable_timing=True)
        e1 = torch.cuda.Event(enable_timing=True)
        e0.record()
        for _ in range(n):
            step()
        e1.record()
        torch.cuda.synchronize(dev)
        t = torch.tensor([e0.elapsed_time(e1) / n], device=dev, dtype=torch.float64)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        return float(t.item()), n

    # parity: both exchanges against one GPU's decode of the whole cache
    q_full = q
    out_full = va.decode(fmt, *full, q_full, H, L, D, va.suggest_splits(fmt, H, L, D)).float()
    del full
    out_fused = torch.empty(H * D, dtype=torch.float16, device=dev)
    bf = va.DeviceBufs(K, V, sK, sV, q, out_fused, ws)
    got_nccl = SplitL.decode(sl, pfn).float()
    got_p2p = sl.decode_peer(pfn, out).float().clone()
    got_fused = sl.decode_fused(fmt, bf, S).float().clone()
    torch.cuda.synchronize(dev)

    def check(got):
        err = (got - out_full).abs()
        ok = bool((err <= 2e-3 + 1e-3 * out_full.abs()).all())
        t = torch.tensor([float(err.max()), 0.0 if ok else 1.0], device=dev, dtype=torch.float64)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        return float(t[0]), t[1].item() == 0.0

    err_nccl, ok_nccl = check(got_nccl)
    err_p2p, ok_p2p = check(got_p2p)
    err_fused, ok_fused = check(got_fused)
    def timed_graph(n=100):
        # the one-launch step counts its epochs on the device, so n steps go
        # into one CUDA graph; every rank replays its own graph, the steps
        # pair up through the peer flags
        st = torch.cuda.Stream(device=dev)
        st.wait_stream(torch.cuda.current_stream(dev))
        with torch.cuda.stream(st):
            for _ in range(5):
                sl.decode_fused(fmt, bf, S, st)
        torch.cuda.synchronize(dev)
        gph = torch.cuda.CUDAGraph()
        with torch.cuda.graph(gph, stream=st):
            for _ in range(n):
                sl.decode_fused(fmt, bf, S, st)
        torch.cuda.synchronize(dev)
        dist.barrier()
        e0 = torch.cuda.Event(enable_timing=True)
        e1 = torch.cuda.Event(enable_timing=True)
        with torch.cuda.stream(st):
            e0.record(st)
            gph.replay()
            e1.record(st)
        torch.cuda.synchronize(dev)
        t = torch.tensor([e0.elapsed_time(e1) / n], device=dev, dtype=torch.float64)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        return float(t.item())

    ms_nccl, n = timed(lambda: SplitL.decode(sl, pfn))
    ms_p2p, _ = timed(lambda: sl.decode_peer(pfn, out))
    ms_fused_eager, _ = timed(lambda: sl.decode_fused(fmt, bf, S))
    ms_fused = timed_graph()
    err_graph, ok_graph = check(out_fused.float())  # the last replayed step's output
    return {"workload": f"split-L decode, one sequence, H={H} D={D} L={L} {fmt} over {world} GPUs",
            "ms": ms_fused, "tok_s": 1e3 / ms_fused, "gbs": algorithmic_bytes(fmt, L) / (ms_fused * 1e6),
            "exchange": "peer-memory exchange and merge fused into the decode (va_decode_splitl, 1 launch per step)",
            "timing": "fused steps replayed from a CUDA graph of 100 (max over ranks); the other variants are "
                      "eager launches from Python",
            "ms_fused_eager": ms_fused_eager, "ms_peer_2launch": ms_p2p, "ms_nccl_allgather": ms_nccl, "steps": n,
            "scaling": "strong",
            "launches_per_step": 1, "local_rows_per_head": Lr, "splits": S,
            "parity": {"against": "1-GPU decode of the same seeded full cache", "tol": "2e-3 + 1e-3*|ref|",
                       "max_err_fused": err_fused, "ok_fused": ok_fused, "max_err_fused_graph": err_graph,
                       "ok_fused_graph": ok_graph, "max_err_peer": err_p2p, "ok_peer": ok_p2p,
                       "max_err_nccl": err_nccl, "ok_nccl": ok_nccl}}


def splitl_base_leg(va, torch, dev, steps, fmt, L=131072):
    """The N=1 base of config 3: the whole sequence on one GPU (strong-scaling
    reference point for splitl_config3 at N > 1)."""
    ms, S, copies, _ = time_format(va, torch, fmt, L, max(50, min(steps, 500)), 3, dev, None, 777, soak_s=0.0)
    return {"workload": f"decode, one sequence, H={H} D={D} L={L} {fmt} on 1 GPU", "ms": ms, "tok_s": 1e3 / ms,
            "gbs": algorithmic_bytes(fmt, L) / (ms * 1e6), "splits": S, "copies": copies}


def run_ours(args, rank, world):
    import torch
    import voltattn_b200 as va
    local = int(os.environ.get("LOCAL_RANK", "0"))
    dev = torch.device("cuda", local)
    torch.cuda.set_device(dev)
    dist = None
    if world > 1:
        # keep NCCL's version banner off stdout: rank 0's stdout carries the JSON line
        if os.environ.get("NCCL_DEBUG", "VERSION").upper() == "VERSION":
            os.environ["NCCL_DEBUG"] = "WARN"
        import torch.distributed as tdist
        tdist.init_process_group("nccl", device_id=dev)
        dist = tdist
    peaks, peaks_kind = measured_peaks()
    fmt, L, K, W = args.fmt, args.L, args.steps, args.warmup
    seed = 1234 + 7919 * rank
    probe = va.probe_ceiling(local, nbytes=4 << 30, reps=10)
    uuid = None
    try:
        uuid = "GPU-" + str(torch.cuda.get_device_properties(dev).uuid)
    except Exception:
        uuid = None

    table = {}
    for f in [x for x in args.table.split(",") if x]:
        if f == fmt:
            continue
        steps_f = max(200, min(K, 5000))
        ms, S_f, copies_f, _ = time_format(va, torch, f, L, steps_f, W, dev, dist, seed, soak_s=0.05)
        gbs = algorithmic_bytes(f, L) / (ms * 1e6)
        table[f] = {"ms": ms, "gbs": gbs, "mbu_probe": gbs / probe, "tok_s": 1e3 / ms, "splits": S_f}
        torch.cuda.empty_cache()

    with ClockSampler(uuid) as clk:
        ms, S, copies, launches = time_format(va, torch, fmt, L, K, W, dev, dist, seed)
    clocks = clk.summary()
    nbytes = algorithmic_bytes(fmt, L)
    gbs = nbytes / (ms * 1e6)
    table[fmt] = {"ms": ms, "gbs": gbs, "mbu_probe": gbs / probe, "tok_s": 1e3 / ms, "splits": S}
    base = table.get("f16+")
    for f, r in table.items():
        if base:
            r["vs_f16+"] = base["ms"] / r["ms"]
        if "f16" in table:
            r["vs_f16"] = table["f16"]["ms"] / r["ms"]
    torch.cuda.empty_cache()
    e2e = e2e_leg(va, torch, fmt, L, K, dev, dist, seed)
    extra = {}
    if not args.no_extra:
        if world == 1:
            extra["gqa_config5"] = gqa_leg(va, torch, dev, K)
            torch.cuda.empty_cache()
            extra["gqa_config5_paged"] = paged_leg(va, torch, dev, K)
            torch.cuda.empty_cache()
            for pf in ("q4+", "f16+"):
                extra[f"prefill_{pf}"] = prefill_leg(va, torch, dev, pf)
                torch.cuda.empty_cache()
            extra["prefill_q4+_unstaged"] = prefill_leg(va, torch, dev, "q4+", staged=False)
            torch.cuda.empty_cache()
            for sf in ("q4+", "q3+"):
                extra[f"splitl_config3_base_{sf}"] = splitl_base_leg(va, torch, dev, K, sf)
                torch.cuda.empty_cache()
            extra["accuracy_config1"] = accuracy_leg(va, torch, dev)
            torch.cuda.empty_cache()
            if not args.no_sweep:
                extra["sweep_config4"] = sweep_leg(va, torch, dev, probe)
                torch.cuda.empty_cache()
        else:
            for sf in ("q4+", "q3+"):
                extra[f"splitl_config3_{sf}"] = splitl_leg(va, torch, dev, dist, world, K, fmt=sf)
                torch.cuda.empty_cache()
            extra["gqa_config5_sharded"] = gqa_sharded_leg(va, torch, dev, dist, world, rank, K)
            torch.cuda.empty_cache()
    cpu = None
    if rank == 0 and world == 1 and not args.no_cpu:
        cpu = cpu_baseline_leg(L, fmt)
    if rank == 0:
        value = world * 1e3 / ms
        traffic = NCU_TRAFFIC_BYTES.get(fmt)
        line = {
            "metric": f"decode tok/s (batch 1, H={H}, D={D}, L={L}, {fmt})",
            "value": value, "unit": "tok/s", "n_gpus": world, "steps": K, "warmup": W, "ms_per_step": ms,
            "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "f32",
            "data": "synthetic: fp32 N(0,1) K/V drawn on the GPU from a seed and packed by the GPU quantizer; "
                    "fp16 N(0,1) q",
            "config": {"workload": f"batch-1 decode H={H} D={D} L={L} fmt={fmt}", "H": H, "D": D, "L": L,
                       "fmt": fmt, "splits": S, "parallelism": f"weak: one sequence per GPU x{world}",
                       "l2": f"rotating {copies} cache copies ({copies * nbytes / 1e6:.0f} MB > 4x L2)",
                       "timing": "CUDA graphs of back-to-back decodes, CUDA events on the launch stream"},
            "impl": "ours",
            "mbu_probe": gbs / probe, "probe_gbs": probe,
            "roofline": {"bound": "hbm", "achieved": gbs, "peak": peaks["hbm_gbs"], "unit": "GB/s",
                         "frac": gbs / peaks["hbm_gbs"], "traffic": traffic,
                         "peak_kind": f"{peaks_kind} (copy bandwidth, MEASURED_PEAKS.json)",
                         "algorithmic_bytes_per_launch": nbytes},
            "cpu_baseline": cpu,
            "e2e": e2e,
            "gpu_launches": K * launches,
            "clocks": clocks,
            "formats": table,
            "extra": extra,
        }
        print(json.dumps(line), flush=True)
    if dist:
        dist.barrier()
        dist.destroy_process_group()


def run_timeline(args):
    """Per-CTA event timeline of the tile kernel (the library built by `make
    timeline`, -DVA_TC_TIMELINE): for --fmt at --L (and L=1024), one decode
    after a decode of another cache copy (single: synchronised between them)
    and the last of three back-to-back decodes (b2b). Times in us from the
    first CTA's start: CTA start, producer start, stages 0..3 landed (as the
    consumers see them), last tile consumed, consumers done, ticket warp done,
    the last head's merge written. Percentiles 0/10/50/90/100 over CTAs."""
    import ctypes
    tl = os.path.join(ROOT, "voltattn_b200", "_build", "timeline")
    if not os.path.exists(os.path.join(tl, "voltattn_b200", "libvoltattn_b200.so")):
        sys.exit("build it first: make timeline")
    sys.path.insert(0, tl)
    import torch
    import voltattn_b200 as va
    lib = va.lib()
    lib.va_debug_tc_timeline.argtypes = [ctypes.c_void_p, ctypes.c_size_t]
    dev = torch.device("cuda", 0)
    buf = np.zeros(1024 * 16, dtype=np.uint64)
    slots = {"start": 0, "producer_start": 11, "stage0": 2, "stage1": 8, "stage2": 9, "stage3": 10,
             "last_tile": 3, "consumers_done": 7, "ticket_done": 4}
    res = {}
    for L in sorted({1024, args.L}):
        caches = [make_cache(va, torch, args.fmt, L, 99 + i, dev) for i in range(3)]
        q = torch.randn(H * D, device=dev).half()
        out = torch.empty(H * D, dtype=torch.float16, device=dev)
        S = va.suggest_splits(args.fmt, H, L, D)
        ws = va.new_workspace(H, D, S, dev)
        bs = [va.DeviceBufs(*c, q, out, ws) for c in caches]
        torch.cuda.synchronize(dev)
        for mode in ("single", "b2b"):
            for _ in range(4):
                va.launch(args.fmt, bs[0], H, L, D, S)
                if mode == "single":
                    torch.cuda.synchronize(dev)
                va.launch(args.fmt, bs[1], H, L, D, S)
                if mode == "b2b":
                    va.launch(args.fmt, bs[2], H, L, D, S)
                torch.cuda.synchronize(dev)
                lib.va_debug_tc_timeline(buf.ctypes.data, buf.nbytes)
            t = buf.reshape(1024, 16).astype(np.int64)
            t = t[: int((t[:, 0] > 0).sum())]
            t0 = t[:, 0].min()
            r = {"ctas": len(t), "splits": S}
            for name, c in slots.items():
                v = t[:, c]
                if (v > 0).all():
                    r[name] = np.percentile((v - t0) / 1e3, [0, 10, 50, 90, 100]).round(2).tolist()
            m = t[:, 5][t[:, 5] > 0]
            r["last_merge"] = round(float((m.max() - t0) / 1e3), 2) if len(m) else None
            res[f"{args.fmt} L={L} {mode}"] = r
        del caches, bs
        torch.cuda.empty_cache()
    print(json.dumps({"timeline": res, "device_error": va.device_error()}), flush=True)


def run_profile(args):
    """Small fixed workload for ncu captures: W warm-up then K decodes of one
    cache (size it above the 126 MB L2 with --L)."""
    import torch
    import voltattn_b200 as va
    dev = torch.device("cuda", 0)
    fmt, L = args.fmt, args.L
    if args.prefill_lq > 0:
        Hq, Hkv, Lq = 32, 8, args.prefill_lq
        b = make_prefill(va, torch, dev, fmt, Hq, Hkv, max(L, Lq), Lq, 5150)
        b.ws = torch.empty(va.prefill_workspace_bytes(Hkv, max(L, Lq), D), dtype=torch.uint8, device=dev)
        for _ in range(args.warmup + args.steps):
            va.prefill(fmt, b, Hq, Hkv, max(L, Lq), Lq, D)
        torch.cuda.synchronize()
        print(json.dumps({"profile": fmt, "prefill_lq": Lq, "L": max(L, Lq),
                          "launches": args.warmup + args.steps, "device_error": va.device_error()}))
        return
    if args.gqa_batch > 0:
        B, Hq, Hkv, Lmax, S = args.gqa_batch, 32, 8, 32768, 4
        b, lens_d, nbytes = make_gqa(va, torch, dev, 4242, fmt, B, Hq, Hkv, Lmax, S)
        for _ in range(args.warmup + args.steps):
            va.decode_gqa(fmt, b, lens_d, B, Hq, Hkv, Lmax, D, S)
        torch.cuda.synchronize()
        print(json.dumps({"profile": fmt, "gqa_batch": B, "bytes": nbytes, "splits": S,
                          "launches": args.warmup + args.steps, "device_error": va.device_error()}))
        return
    cache = make_cache(va, torch, fmt, L, 99, dev)
    q = torch.randn(H * D, device=dev).half()
    out = torch.empty(H * D, dtype=torch.float16, device=dev)
    S = va.suggest_splits(fmt, H, L, D)
    ws = va.new_workspace(H, D, S, dev)
    b = va.DeviceBufs(*cache, q, out, ws)
    for _ in range(args.warmup + args.steps):
        va.launch(fmt, b, H, L, D, S)
    torch.cuda.synchronize()
    print(json.dumps({"profile": fmt, "L": L, "splits": S, "launches": args.warmup + args.steps,
                      "device_error": va.device_error()}))


def main():
    args = parse_args()
    if args.timeline:
        run_timeline(args)
        return
    if args.profile:
        run_profile(args)
        return
    rank = int(os.environ.get("RANK", "0"))
    world = int(os.environ.get("WORLD_SIZE", "1"))
    if args.impl == "reference":
        run_reference_arm(args, rank)
        return
    run_ours(args, rank, world)


if __name__ == "__main__":
    main()
