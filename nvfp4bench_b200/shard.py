"""N-sharding of the GEMM across ranks (one process per GPU).

D = A * B^T is split along N: rank r owns weight rows [n0, n1) of B (and the matching
columns of D); A is replicated. The GEMM needs no communication; the only collective is the
max-over-ranks reduction of step times (and, optionally, an all-gather of the D shards:
NCCL after the GEMM, or fused into the GEMM epilogue through GatheredOutput).
"""
from __future__ import annotations

from typing import Tuple


def shard_bounds(n_total: int, world: int, rank: int, align: int = 128) -> Tuple[int, int]:
    """Contiguous [n0, n1) slice of n_total rows for `rank`, in whole `align`-row blocks
    (the kernels' tile height) except for the last rank, which takes the remainder."""
    if world < 1 or not 0 <= rank < world:
        raise ValueError("bad world/rank")
    blocks = (n_total + align - 1) // align
    b0 = blocks * rank // world
    b1 = blocks * (rank + 1) // world
    return min(b0 * align, n_total), min(b1 * align, n_total)


def max_over_ranks(values, device=None):
    """Element-wise max of a list of floats over all ranks (identity without a process group)."""
    import torch
    import torch.distributed as dist
    t = torch.tensor(list(values), dtype=torch.float64, device=device)
    if dist.is_available() and dist.is_initialized() and dist.get_world_size() > 1:
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
    return t.tolist()


def gather_shards(local, n_total: int, out=None):
    """One all-gather of the per-rank column shards [M][n1-n0] into [world][M][width] (rank r's
    shard in slot r, padded to the widest shard): the single NVLink exchange."""
    import torch
    import torch.distributed as dist
    world = dist.get_world_size()
    M = local.shape[0]
    spans = [shard_bounds(n_total, world, r) for r in range(world)]
    width = max(n1 - n0 for n0, n1 in spans)  # collectives want equal sizes: pad, then trim
    if local.shape[1] == width:
        padded = local.contiguous()
    else:
        padded = torch.zeros((M, width), dtype=local.dtype, device=local.device)
        padded[:, : local.shape[1]] = local
    if out is None:
        out = torch.empty((world, M, width), dtype=local.dtype, device=local.device)
    dist.all_gather_into_tensor(out.view(world * M, width), padded)
    return out


def shards_to_row_major(shards, n_total: int, out=None):
    """[world][M][width] shards -> row-major [M][n_total] (the optional 2-D copy)."""
    import torch
    world, M, width = shards.shape
    spans = [shard_bounds(n_total, world, r) for r in range(world)]
    if out is None:
        out = torch.empty((M, n_total), dtype=shards.dtype, device=shards.device)
    for r, (n0, n1) in enumerate(spans):
        out[:, n0:n1].copy_(shards[r, :, : n1 - n0])
    return out


def gather_columns(local, n_total: int, device=None):
    """All-gather of per-rank column shards [M][n1-n0] into the full [M][n_total] matrix."""
    return shards_to_row_major(gather_shards(local, n_total), n_total)


class GatheredOutput:
    """The all-gathered output, written by the GEMMs themselves: every rank holds a row-major
    [M][n_total] buffer; rank r's GEMM computes its column shard [n0, n1) and its epilogue
    stores each finished tile into its own buffer and, over NVLink, into every other rank's
    (CUDA IPC mappings of the peers' buffers, exchanged once through the process group). The
    fused counterpart of gather_columns: no separate collective and no reordering copy.

    Use: g = GatheredOutput(M, n_total, torch.bfloat16, device); each step
    api.gemm(..., N=g.n1 - g.n0, out=g.local, peers=g.peers); then g.wait_all() before reading
    g.full (it orders every rank's GEMM before the read) and before the next step's GEMM writes
    into buffers that peers may still read."""

    def __init__(self, M: int, n_total: int, dtype, device, group=None):
        import torch
        import torch.distributed as dist
        from nvfp4bench_b200 import api
        self.group = group
        self.world = dist.get_world_size(group)
        self.rank = dist.get_rank(group)
        self.n0, self.n1 = shard_bounds(n_total, self.world, self.rank)
        esize = torch.empty((), dtype=dtype).element_size()
        if (n_total * esize) % 16 or (self.n0 * esize) % 16:
            raise ValueError("rows and shard starts must be 16-byte aligned for the TMA stores")
        self.full = torch.empty((M, n_total), dtype=dtype, device=device)
        self.local = self.full[:, self.n0:self.n1]
        handle = api.ipc_handle(self.full)
        handles = [None] * self.world
        dist.all_gather_object(handles, handle, group=group)
        self._bases = []
        for r, (h, off) in enumerate(handles):
            if r != self.rank:
                self._bases.append(api.ipc_open(h, off))
        # Each peer's buffer at this rank's shard: addressed exactly like `local`.
        self.peers = [b + self.n0 * esize for b in self._bases]
        self._flag = None

    def wait_all(self) -> None:
        """Every rank's GEMM writes (into every buffer) are complete and visible here. With
        NCCL a one-word all-reduce orders them on the device; otherwise the host synchronises
        and meets the other ranks at a barrier."""
        import torch
        import torch.distributed as dist
        if dist.get_backend(self.group) == "nccl":
            if self._flag is None:
                self._flag = torch.zeros(1, dtype=torch.int32, device=self.full.device)
            dist.all_reduce(self._flag, group=self.group)
        else:
            if self.full.is_cuda:
                torch.cuda.synchronize(self.full.device)
            dist.barrier(group=self.group)

    def close(self) -> None:
        """Unmap the peers' buffers (after every rank's last GEMM: call wait_all first)."""
        from nvfp4bench_b200 import api
        for b in self._bases:
            api.ipc_close(b)
        self._bases, self.peers = [], []
