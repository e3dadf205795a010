"""CPU: the N-sharding host logic with 2 gloo ranks (no GPU)."""
import os
import socket

import numpy as np
import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

from nvfp4bench_b200.shard import gather_columns, max_over_ranks, shard_bounds


def test_shard_bounds_cover_disjoint():
    for n_total in (1, 127, 128, 4096, 14336, 65536, 1000):
        for world in (1, 2, 3, 4, 8):
            spans = [shard_bounds(n_total, world, r) for r in range(world)]
            assert spans[0][0] == 0 and spans[-1][1] == n_total
            for (a0, a1), (b0, b1) in zip(spans, spans[1:]):
                assert a1 == b0 and a0 <= a1
            for n0, _ in spans:
                assert n0 % 128 == 0


def _free_port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    p = s.getsockname()[1]
    s.close()
    return p


def _worker(rank, world, port, out_q):
    import oracle
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world)
    M, N, K = 8, 300, 64
    a = oracle.make_uniform(M, K, 1234)
    b = oracle.make_uniform(N, K, 1234 ^ 0xABCDEF)
    pa, sa = oracle.quantize(a)
    pb, sb = oracle.quantize(b)
    adq, bdq = oracle.dequantize(pa, sa, K), oracle.dequantize(pb, sb, K)
    n0, n1 = shard_bounds(N, world, rank)
    local = torch.from_numpy(oracle.gemm_nt(adq, bdq[n0:n1]))
    full = gather_columns(local, N)
    t = max_over_ranks([float(rank + 1), 10.0 - rank])
    if rank == 0:
        out_q.put((full.numpy(), oracle.gemm_nt(adq, bdq), t))
    dist.barrier()
    dist.destroy_process_group()


def test_sharded_gemm_equals_unsharded_two_gloo_ranks():
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, 2, port, q)) for r in range(2)]
    for p in procs:
        p.start()
    full, ref, t = q.get(timeout=120)
    for p in procs:
        p.join(timeout=60)
        assert p.exitcode == 0
    assert np.array_equal(full, ref)  # column shards are independent: exact
    assert t == [2.0, 10.0]


def _gathered_worker(rank, world, port, out_q):
    """GatheredOutput's host side with the CUDA IPC calls faked: each rank 'exports' its
    buffer as its rank number and 'maps' peer r at a synthetic address; the peer destinations
    handed to the GEMM must be those addresses plus this rank's shard offset."""
    from nvfp4bench_b200 import api
    from nvfp4bench_b200.shard import GatheredOutput
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world)
    opened, closed = [], []
    api.ipc_handle = lambda t: (bytes([rank]) * api.IPC_HANDLE_BYTES, 256 * rank)
    api.ipc_open = lambda h, off: opened.append((h[0], off)) or (0x100000 * (h[0] + 1) + off)
    api.ipc_close = lambda p: closed.append(p)
    go = GatheredOutput(64, 1280, torch.bfloat16, "cpu")
    peers = list(go.peers)
    go.wait_all()
    go.close()
    out_q.put((rank, go.n0, go.n1, tuple(go.local.stride()), go.local.data_ptr() - go.full.data_ptr(),
               peers, opened, closed))
    dist.barrier()
    dist.destroy_process_group()


def test_gathered_output_peer_addresses_three_gloo_ranks():
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    world = 3
    procs = [ctx.Process(target=_gathered_worker, args=(r, world, port, q)) for r in range(world)]
    for p in procs:
        p.start()
    res = sorted(q.get(timeout=120) for _ in procs)
    for p in procs:
        p.join(timeout=60)
        assert p.exitcode == 0
    spans = [shard_bounds(1280, world, r) for r in range(world)]
    for rank, n0, n1, stride, off, peers, opened, closed in res:
        assert (n0, n1) == spans[rank]
        assert stride == (1280, 1) and off == 2 * n0  # the local slice of the row-major buffer
        others = [r for r in range(world) if r != rank]
        assert opened == [(r, 256 * r) for r in others]
        bases = [0x100000 * (r + 1) + 256 * r for r in others]
        assert peers == [b + 2 * n0 for b in bases]
        assert closed == bases
