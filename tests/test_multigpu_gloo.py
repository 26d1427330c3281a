"""Multi-rank host logic of voltattn_b200.launcher on CPU (gloo, world size 2):
the split-L partition, the partial all-gather and the combine order, head-block
gathering, and failure of a rank surfacing as an error on the others (no
hang). The per-rank compute is the oracle's partial / combine; the GPU kernels
of the same steps are covered by tests/test_gpu_decode.py."""
import os
import socket
import tempfile

import numpy as np
import pytest
import torch.multiprocessing as mp


def free_port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    p = s.getsockname()[1]
    s.close()
    return p


def _init(rank, world, port, timeout_s=30.0):
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    os.environ["RANK"] = str(rank)
    os.environ["WORLD_SIZE"] = str(world)
    from voltattn_b200.launcher import init_distributed
    return init_distributed("gloo", timeout_s=timeout_s)


def _split_l_worker(rank, world, port, outdir):
    import torch
    import torch.distributed as dist
    from oracle.oracle import Oracle
    from voltattn_b200.launcher import SplitL
    _init(rank, world, port)
    o = Oracle()
    H, L, D = 4, 1003, 64
    kx, vx, q = o.gen_case(55, H, L, D)
    kd, vd = o.round_to_half(kx), o.round_to_half(vx)
    sl = SplitL(L)

    def partial_fn(j0, j1):
        return torch.from_numpy(np.stack([o.partial(kd, vd, q, H, L, D, h, j0, j1) for h in range(H)]))

    def combine_fn(gathered, H_, D_):
        g = gathered.numpy()  # [R][H][1][D+2] -> the reference's [H][S][D+2] slot order
        ws = np.ascontiguousarray(np.transpose(g, (1, 0, 2, 3))).reshape(-1)
        return torch.from_numpy(o.h2f(o.combine(ws, H_, g.shape[0], D_)))

    out = sl.decode(partial_fn, combine_fn)
    np.save(os.path.join(outdir, f"out{rank}.npy"), out.numpy())
    np.save(os.path.join(outdir, f"range{rank}.npy"), np.array([sl.j0, sl.j1]))
    dist.barrier()
    dist.destroy_process_group()


def test_split_l_two_ranks(oracle):
    port = free_port()
    with tempfile.TemporaryDirectory() as d:
        mp.spawn(_split_l_worker, args=(2, port, d), nprocs=2, join=True)
        H, L, D = 4, 1003, 64
        kx, vx, q = oracle.gen_case(55, H, L, D)
        ref = oracle.reference(oracle.round_to_half(kx), oracle.round_to_half(vx), q, H, L, D)
        r0, r1 = np.load(os.path.join(d, "range0.npy")), np.load(os.path.join(d, "range1.npy"))
        assert r0[0] == 0 and r0[1] == r1[0] and r1[1] == L and r0[1] % 8 == 0
        for r in range(2):
            out = np.load(os.path.join(d, f"out{r}.npy"))
            np.testing.assert_allclose(out, ref, atol=2e-3, rtol=1e-3)


def _head_worker(rank, world, port, outdir):
    import torch
    import torch.distributed as dist
    from voltattn_b200.launcher import HeadSharding
    _init(rank, world, port)
    H, D = 5, 8
    hs = HeadSharding(H)
    local = torch.arange(hs.h0 * D, hs.h1 * D, dtype=torch.float32)
    full = hs.gather_output(local, D)
    np.save(os.path.join(outdir, f"heads{rank}.npy"), full.numpy())
    dist.barrier()
    dist.destroy_process_group()


def test_head_sharding_gather():
    port = free_port()
    with tempfile.TemporaryDirectory() as d:
        mp.spawn(_head_worker, args=(2, port, d), nprocs=2, join=True)
        for r in range(2):
            np.testing.assert_array_equal(np.load(os.path.join(d, f"heads{r}.npy")), np.arange(40, dtype=np.float32))


def _failing_worker(rank, world, port, outdir):
    import torch
    from voltattn_b200.launcher import SplitL
    _init(rank, world, port, timeout_s=5.0)
    sl = SplitL(100)
    if rank == 1:
        raise SystemExit(3)  # this rank dies before the gather
    try:
        sl.gather(torch.zeros(2, 10))
        status = "completed"
    except Exception as e:  # noqa: BLE001 — any collective error is the expected outcome
        status = "error:" + type(e).__name__
    with open(os.path.join(outdir, "status"), "w") as fh:
        fh.write(status)


def test_dead_rank_surfaces_as_error():
    port = free_port()
    with tempfile.TemporaryDirectory() as d:
        ctx = mp.spawn(_failing_worker, args=(2, port, d), nprocs=2, join=False)
        try:
            ctx.join(timeout=60)
        except Exception:  # the dead rank's exit is reported here
            pass
        for p in ctx.processes:
            p.join(timeout=60)
            if p.is_alive():
                p.kill()
        with open(os.path.join(d, "status")) as fh:
            assert fh.read().startswith("error:")


def test_split_range_properties():
    from voltattn_b200.launcher import split_range
    for n in [1, 7, 8, 100, 1003, 16384, 65536]:
        for parts in [1, 2, 3, 4, 8]:
            rs = [split_range(n, parts, i) for i in range(parts)]
            assert rs[0][0] == 0 and rs[-1][1] == n
            for a, b in zip(rs, rs[1:]):
                assert a[1] == b[0]
            for a, b in rs[:-1]:
                assert b % 8 == 0 or b == n
    with pytest.raises(ValueError):
        split_range(10, 2, 2)
