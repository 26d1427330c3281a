"""Multi-GPU launcher: one process per GPU, torch.distributed (NCCL) plumbing.

The reference is single-GPU (src/voltattn.cu:803-835 splits the KV length only
inside one GPU). Decode shards three ways:

* by sequence (`BatchSharding`): each rank decodes its own sequences, no
  collective on the data path;
* by head (`HeadSharding`): rank r owns a contiguous block of heads; the fp16
  outputs are all-gathered when every rank needs the full output;
* by KV length (`SplitL`): rank r holds a contiguous range of every head's
  positions, decodes it into per-head (m, l, o[D]) partials
  (va_decode_partial), the partials (H*(D+2) floats per rank, ~16.6 KB at
  H=32) are all-gathered over NCCL into this GPU's own memory, and the
  log-sum-exp combine (va_combine_partials) produces the output on every
  rank. This is the reference's split-L combine (src/voltattn.cu:651-672)
  lifted across GPUs. `SplitLPeer` replaces the NCCL gather by one fused
  kernel over NVLink peer memory (epoch-tagged 64-bit stores into the peers'
  buffers, no flags, no TMA and no multicast).

The local compute is injectable so that the collective orchestration can be
tested on CPU with the gloo backend.
"""
from __future__ import annotations

import datetime
import os
from typing import Callable, Optional, Sequence, Tuple

import torch
import torch.distributed as dist


def init_distributed(backend: Optional[str] = None, timeout_s: float = 60.0) -> Tuple[int, int]:
    """Initialises the default process group from torchrun's environment
    (RANK, WORLD_SIZE, MASTER_ADDR, MASTER_PORT, LOCAL_RANK). A rank that
    never joins, or dies before a collective, makes the others fail with an
    error after `timeout_s` instead of hanging."""
    if dist.is_initialized():
        return dist.get_rank(), dist.get_world_size()
    if backend is None:
        backend = "nccl" if torch.cuda.is_available() else "gloo"
    kwargs = {"backend": backend, "timeout": datetime.timedelta(seconds=timeout_s)}
    if backend == "nccl":
        local = int(os.environ.get("LOCAL_RANK", "0"))
        torch.cuda.set_device(local)
        kwargs["device_id"] = torch.device("cuda", local)
    dist.init_process_group(**kwargs)
    return dist.get_rank(), dist.get_world_size()


def split_range(n: int, parts: int, idx: int, align: int = 8) -> Tuple[int, int]:
    """Contiguous, balanced share [j0, j1) of n items for part idx of parts;
    interior boundaries fall on multiples of `align` where n allows (whole
    8-row blocks keep every rank's bulk copies aligned)."""
    if parts < 1 or not 0 <= idx < parts:
        raise ValueError("bad partition")

    def bound(k: int) -> int:
        if k <= 0:
            return 0
        if k >= parts:
            return n
        b = (n * k) // parts
        b = ((b + align // 2) // align) * align
        return max(0, min(n, b))

    return bound(idx), bound(idx + 1)


class SplitL:
    """KV-length split across the ranks of a process group.

    partial_fn(j0, j1) -> float32 tensor [H][D+2] of this rank's per-head
        partials over its positions (default: the caller passes a closure over
        voltattn_b200.decode_partial on its local cache);
    combine_fn(gathered [R][H][1][D+2], H, D) -> output (default: the
        va_combine_partials kernel, fp16 [H*D] on this rank's GPU).
    """

    def __init__(self, L_total: int, group=None):
        self.group = group
        self.rank = dist.get_rank(group)
        self.world = dist.get_world_size(group)
        self.L_total = L_total
        self.j0, self.j1 = split_range(L_total, self.world, self.rank)

    @property
    def local_len(self) -> int:
        return self.j1 - self.j0

    def gather(self, partial: torch.Tensor) -> torch.Tensor:
        """All-gathers the [H][D+2] partials into [R][H][1][D+2] on this rank."""
        parts = [torch.empty_like(partial) for _ in range(self.world)]
        dist.all_gather(parts, partial.contiguous(), group=self.group)
        g = torch.stack(parts, 0)
        return g.view(self.world, partial.shape[0], 1, partial.shape[1])

    def decode(self, partial_fn: Callable[[int, int], torch.Tensor],
               combine_fn: Optional[Callable[[torch.Tensor, int, int], torch.Tensor]] = None) -> torch.Tensor:
        partial = partial_fn(self.j0, self.j1)
        H, D2 = partial.shape
        gathered = self.gather(partial)
        if combine_fn is None:
            combine_fn = _gpu_combine
        return combine_fn(gathered, H, D2 - 2)


class SplitLPeer(SplitL):
    """SplitL whose partial exchange runs over NVLink peer memory instead of
    NCCL: one fused kernel per step (va_exchange_combine) stores this rank's
    partials into every rank's buffer as epoch-tagged words, waits until the
    peers' words carry the step's epoch and merges them. Buffers come from torch symmetric
    memory (mapped into every rank's address space)."""

    def __init__(self, L_total: int, H: int, D: int, device, group=None):
        super().__init__(L_total, group)
        import torch.distributed._symmetric_memory as symm_mem
        import voltattn_b200 as va
        self.H, self.D = H, D
        nbytes = va.exchange_buffer_bytes(self.world, H, D)
        g = self.group if self.group is not None else dist.group.WORLD
        # two buffers: host-counted steps (decode_peer) and device-counted
        # steps (decode_fused); one buffer must not serve both ways
        self.buf = symm_mem.empty(nbytes, dtype=torch.uint8, device=device)
        self.buf.zero_()
        self.handle = symm_mem.rendezvous(self.buf, g)
        self.peer_ptrs = [int(p) for p in self.handle.buffer_ptrs]
        self.fbuf = symm_mem.empty(nbytes, dtype=torch.uint8, device=device)
        self.fbuf.zero_()
        self.fhandle = symm_mem.rendezvous(self.fbuf, g)
        self.fused_ptrs = [int(p) for p in self.fhandle.buffer_ptrs]
        self.epoch = 0
        torch.cuda.synchronize(device)
        dist.barrier(group=self.group)

    def decode_fused(self, fmt: str, bufs, S: int, stream=None) -> torch.Tensor:
        """One launch per step (va_decode_splitl): the local decode of this
        rank's positions with the peer exchange and merge fused into it;
        bufs.K/V/scales hold this rank's local_len rows per head, the merged
        fp16 output lands in bufs.out on every rank. The steps are counted on
        the device (epoch 0), so calls can be captured in a CUDA graph; this
        object's buffers then serve only this path."""
        import ctypes
        import voltattn_b200 as va
        if not hasattr(self, "_peer_array"):
            self._peer_array = (ctypes.c_void_p * self.world)(*self.fused_ptrs)
        va.decode_splitl(fmt, bufs, self.H, self.local_len, self.D, S, self.world, self.rank, self._peer_array, 0,
                         stream)
        return bufs.out

    def decode_peer(self, partial_fn: Callable[[int, int], torch.Tensor], out: torch.Tensor, stream=None) -> torch.Tensor:
        import voltattn_b200 as va
        partial = partial_fn(self.j0, self.j1)
        self.epoch += 1
        va.exchange_combine(partial, self.H, self.D, self.world, self.rank, self.peer_ptrs, self.epoch, out, stream)
        return out


def _gpu_combine(gathered: torch.Tensor, H: int, D: int) -> torch.Tensor:
    import voltattn_b200 as va
    out = torch.empty(H * D, dtype=torch.float16, device=gathered.device)
    va.combine_partials(gathered.contiguous(), gathered.shape[0], H, 1, D, out)
    return out


class HeadSharding:
    """Contiguous head blocks per rank; `gather_output` all-gathers the fp16
    [h1-h0][D] blocks into the full [H][D] output on every rank."""

    def __init__(self, H: int, group=None):
        self.group = group
        self.rank = dist.get_rank(group)
        self.world = dist.get_world_size(group)
        self.H = H
        self.h0, self.h1 = split_range(H, self.world, self.rank, align=1)
        self.bounds = [split_range(H, self.world, r, align=1) for r in range(self.world)]

    def gather_output(self, local_out: torch.Tensor, D: int) -> torch.Tensor:
        hmax = max(b - a for a, b in self.bounds)
        buf = torch.zeros(hmax * D, dtype=local_out.dtype, device=local_out.device)
        buf[: local_out.numel()] = local_out.reshape(-1)
        parts = [torch.empty_like(buf) for _ in range(self.world)]
        dist.all_gather(parts, buf, group=self.group)
        return torch.cat([parts[r][: (b - a) * D] for r, (a, b) in enumerate(self.bounds)])


class BatchSharding:
    """Sequences per rank; no collective on the data path."""

    def __init__(self, batch: int, group=None):
        self.rank = dist.get_rank(group)
        self.world = dist.get_world_size(group)
        self.b0, self.b1 = split_range(batch, self.world, self.rank, align=1)

    def local(self, seqs: Sequence):
        return seqs[self.b0:self.b1]
