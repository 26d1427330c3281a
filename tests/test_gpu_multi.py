"""Multi-GPU split-L decode on 2 GPUs (skipped with fewer): each rank holds a
contiguous range of every head's KV positions, decodes it into partials, and
the output is assembled (a) with an NCCL all-gather + the combine kernel,
(b) with the peer-memory exchange kernel (va_exchange_combine) and (c) with
the exchange fused into the decode (va_decode_splitl, one launch per step),
over three consecutive steps; all must match the single-cache oracle
reference."""
import os
import socket
import tempfile

import numpy as np
import pytest
import torch.multiprocessing as mp

pytestmark = pytest.mark.gpu

ATOL, RTOL = 2e-3, 1e-3


def _port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    p = s.getsockname()[1]
    s.close()
    return p


def _worker(rank, world, port, outdir):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), RANK=str(rank), WORLD_SIZE=str(world),
                      LOCAL_RANK=str(rank), NCCL_NVLS_ENABLE="0")
    import torch
    import voltattn_b200 as va
    from oracle.oracle import Oracle
    from voltattn_b200.launcher import SplitL, SplitLPeer, init_distributed
    init_distributed("nccl", timeout_s=60)
    dev = torch.device("cuda", rank)
    o = Oracle()
    H, L, D, fmt, bits = 8, 2051, 128, "q4+", 4
    kx, vx, _ = o.gen_case(1234, H, L, D)
    kc, ks = o.quantize(kx, H, L, D, bits)
    vc, vs = o.quantize(vx, H, L, D, bits)
    kd, vd = o.dequant(kc, ks, H, L, D, bits), o.dequant(vc, vs, H, L, D, bits)
    sl = SplitLPeer(L, H, D, dev)
    j0, j1 = sl.j0, sl.j1
    Lr = j1 - j0
    sub = lambda a: np.ascontiguousarray(a.reshape(H, L, D)[:, j0:j1]).reshape(-1)  # noqa: E731
    Kq, sK = o.quantize(sub(kx), H, Lr, D, bits)
    Vq, sV = o.quantize(sub(vx), H, Lr, D, bits)
    K, V = torch.from_numpy(Kq).to(dev), torch.from_numpy(Vq).to(dev)
    sKd = torch.from_numpy(sK).to(dev).view(torch.float16)
    sVd = torch.from_numpy(sV).to(dev).view(torch.float16)
    S = 2
    ws = va.new_workspace(H, D, S, dev)
    partial = torch.empty(H, D + 2, dtype=torch.float32, device=dev)
    results = []
    rng = np.random.default_rng(5)
    for step in range(3):
        q = o.f2h(rng.standard_normal(H * D).astype(np.float32))
        qd = torch.from_numpy(q).to(dev).view(torch.float16)
        out_local = torch.empty(H * D, dtype=torch.float16, device=dev)
        b = va.DeviceBufs(K, V, sKd, sVd, qd, out_local, ws)

        def pfn(a, bnd):
            va.decode_partial(fmt, b, H, Lr, D, S, partial)
            return partial

        ref = o.reference(kd, vd, q, H, L, D)
        out_nccl = SplitL.decode(sl, pfn)
        out_p2p = torch.empty(H * D, dtype=torch.float16, device=dev)
        sl.decode_peer(pfn, out_p2p)
        out_fused = torch.empty(H * D, dtype=torch.float16, device=dev)
        sl.decode_fused(fmt, va.DeviceBufs(K, V, sKd, sVd, qd, out_fused, ws), S)
        torch.cuda.synchronize(dev)
        for name, out in (("nccl", out_nccl), ("p2p", out_p2p), ("fused", out_fused)):
            err = np.abs(out.float().cpu().numpy() - ref)
            results.append((name, step, bool((err <= ATOL + RTOL * np.abs(ref)).all()), float(err.max())))
    results.append(("device_error", -1, va.device_error() == 0, 0.0))
    with open(os.path.join(outdir, f"r{rank}.txt"), "w") as fh:
        fh.write(repr(results))
    torch.distributed.barrier()
    torch.distributed.destroy_process_group()


def test_split_l_two_gpus():
    import torch
    if torch.cuda.device_count() < 2:
        pytest.skip("needs 2 GPUs")
    with tempfile.TemporaryDirectory() as d:
        mp.spawn(_worker, args=(2, _port(), d), nprocs=2, join=True)
        for r in range(2):
            res = eval(open(os.path.join(d, f"r{r}.txt")).read())  # noqa: S307 — our own repr
            bad = [x for x in res if not x[2]]
            assert not bad, res
