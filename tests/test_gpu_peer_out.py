"""GPU: output pitch (ldc) and peer destinations (the fused all-gather of a column-sharded
GEMM). Every destination must hold exactly the bytes of the plain GEMM's output; nothing
outside the written column slice may change."""
import os
import socket

import pytest
import torch

from gpu_helpers import make_operand, run_gemm

pytestmark = pytest.mark.gpu


CASES = [
    ((256, 512, 1024), dict(cta_group=1, tile_n=128), torch.bfloat16),
    ((300, 640, 320), dict(cta_group=1, tile_n=256), torch.bfloat16),
    ((512, 512, 512), dict(cta_group=2), torch.float32),
    ((16, 1024, 512), {}, torch.bfloat16),  # decode-sized: routed to the general kernel
]


def ref_kw(kw):
    # A pitch or peers take decode-sized problems to the general kernel (one-SM, 128-wide
    # tiles at this size) instead of the split-K weight-streaming kernel, whose sums are
    # ordered differently: the reference run takes the same kernel.
    return kw or dict(cta_group=1, tile_n=128)


@pytest.mark.parametrize("shape,kw,dtype", CASES)
def test_column_slice_output(api, shape, kw, dtype):
    """out = a column slice [:, 128:128+N] of a wider matrix: row pitch = its stride."""
    M, N, K = shape
    _, a = make_operand(api, M, K, 11)
    _, b = make_operand(api, N, K, 12)
    ref = run_gemm(api, a, b, M, N, K, out_dtype=dtype, **ref_kw(kw))
    wide = torch.full((M, N + 256), -7.0, dtype=dtype, device="cuda")
    api.gemm(a.packed, a.scales_tc, b.packed, b.scales_tc, M, N, K, wide[:, 128:128 + N], **kw)
    torch.cuda.synchronize()
    assert api.device_error() == 0
    assert torch.equal(wide[:, 128:128 + N], ref)
    assert bool((wide[:, :128] == -7.0).all()) and bool((wide[:, 128 + N:] == -7.0).all())


@pytest.mark.parametrize("shape,kw,dtype", CASES)
def test_peer_destinations_receive_every_tile(api, shape, kw, dtype):
    """Two further destinations on the same GPU stand in for peers: each must equal the
    output, slice for slice."""
    M, N, K = shape
    n_total = N + 256
    _, a = make_operand(api, M, K, 13)
    _, b = make_operand(api, N, K, 14)
    ref = run_gemm(api, a, b, M, N, K, out_dtype=dtype, **ref_kw(kw))
    bufs = [torch.full((M, n_total), 3.0, dtype=dtype, device="cuda") for _ in range(3)]
    esize = bufs[0].element_size()
    peers = [bb.data_ptr() + 128 * esize for bb in bufs[1:]]
    api.gemm(a.packed, a.scales_tc, b.packed, b.scales_tc, M, N, K, bufs[0][:, 128:128 + N],
             peers=peers, **kw)
    torch.cuda.synchronize()
    assert api.device_error() == 0
    for bb in bufs:
        assert torch.equal(bb[:, 128:128 + N], ref)
        assert bool((bb[:, :128] == 3.0).all()) and bool((bb[:, 128 + N:] == 3.0).all())


def test_peer_destinations_sparse_kernel(api):
    M, N, K = 256, 512, 1024
    x = api.fill_normal(M, K, 21)
    meta = api.sparse_meta(M, K, 0x24)
    api.sparse_prune(x, meta)
    ta = api.quantize_block(x, 32)
    vals = api.sparse_compress(ta.packed, meta, K)
    tb = api.quantize_block(api.fill_normal(N, K, 22), 32)
    ref = torch.empty((M, N), dtype=torch.bfloat16, device="cuda")
    api.gemm(vals, ta.scales_tc, tb.packed, tb.scales_tc, M, N, K, ref, mode=api.MODE_SPARSE24,
             a_meta=meta)
    out = torch.empty_like(ref)
    peer = torch.zeros_like(ref)
    api.gemm(vals, ta.scales_tc, tb.packed, tb.scales_tc, M, N, K, out, mode=api.MODE_SPARSE24,
             a_meta=meta, peers=[peer.data_ptr()])
    torch.cuda.synchronize()
    assert api.device_error() == 0
    assert torch.equal(out, ref) and torch.equal(peer, ref)


def test_peer_destinations_rejected_without_tma_store_path(api):
    M, N, K = 128, 256, 256
    _, a = make_operand(api, M, K, 1)
    _, b = make_operand(api, N, K, 2)
    peer = torch.empty((M, N), dtype=torch.bfloat16, device="cuda")
    pk = torch.empty((M, N // 2), dtype=torch.uint8, device="cuda")
    sc = torch.empty((M, N // 16), dtype=torch.uint8, device="cuda")
    with pytest.raises(api.Nvfp4Error, match="peer"):
        api.gemm(a.packed, a.scales_tc, b.packed, b.scales_tc, M, N, K, pk, out_scales=sc,
                 peers=[peer.data_ptr()])
    out = torch.empty((M, N), dtype=torch.bfloat16, device="cuda")
    with pytest.raises(api.Nvfp4Error, match="aligned"):
        api.gemm(a.packed, a.scales_tc, b.packed, b.scales_tc, M, N, K, out,
                 peers=[peer.data_ptr() + 2])
    with pytest.raises(api.Nvfp4Error, match="n_peers"):
        api.gemm(a.packed, a.scales_tc, b.packed, b.scales_tc, M, N, K, out,
                 peers=[peer.data_ptr()] * 8)
    with pytest.raises(api.Nvfp4Error, match="no-alloc"):
        args = api.gemm_args(a.packed, a.scales, b.packed, b.scales, M, N, K, out,
                             sf_layout=api.SF_CANONICAL, peers=[peer.data_ptr()])
        api._call(api.lib().nvfp4_b200_gemm_noalloc, api.C.byref(args), api._stream(None))
    assert api.device_error() == 0


def test_ipc_roundtrip_in_process(api):
    """Export and reference-count bookkeeping; opening needs another process (below)."""
    t = torch.empty(1 << 20, dtype=torch.uint8, device="cuda")
    view = t[4096:]
    h, off = api.ipc_handle(view)
    assert len(h) == api.IPC_HANDLE_BYTES
    h0, off0 = api.ipc_handle(t)
    assert off - off0 == 4096
    with pytest.raises(api.Nvfp4Error, match="not returned"):
        api.ipc_close(view.data_ptr())


def _free_port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    p = s.getsockname()[1]
    s.close()
    return p


def _ipc_worker(rank, world, port, q):
    import sys
    sys.path.insert(0, os.path.dirname(os.path.dirname(os.path.abspath(__file__))))
    import torch.distributed as dist
    from nvfp4bench_b200 import api
    from nvfp4bench_b200.shard import GatheredOutput, shard_bounds
    try:
        os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
        dist.init_process_group("gloo", rank=rank, world_size=world)
        torch.cuda.set_device(0)
        M, n_total, K = 384, 1280, 512
        a = api.quantize(api.fill_normal(M, K, 31))
        b_full = api.fill_normal(n_total, K, 32)
        n0, n1 = shard_bounds(n_total, world, rank)
        b = api.quantize(b_full[n0:n1].contiguous())
        go = GatheredOutput(M, n_total, torch.bfloat16, "cuda")
        go.full.fill_(5.0)
        go.wait_all()
        api.gemm(a.packed, a.scales_tc, b.packed, b.scales_tc, M, n1 - n0, K, go.local,
                 tile_n=128, cta_group=1, peers=go.peers)
        go.wait_all()
        bf = api.quantize(b_full)
        ref = torch.empty((M, n_total), dtype=torch.bfloat16, device="cuda")
        api.gemm(a.packed, a.scales_tc, bf.packed, bf.scales_tc, M, n_total, K, ref, tile_n=128,
                 cta_group=1)
        torch.cuda.synchronize()
        ok = bool(torch.equal(go.full, ref)) and api.device_error() == 0
        go.wait_all()
        go.close()
        dist.barrier()
        dist.destroy_process_group()
        q.put((rank, ok, ""))
    except Exception as e:  # reported to the parent
        q.put((rank, False, repr(e)))


def test_gathered_output_two_processes_one_gpu(api):
    """Two ranks (processes) on one GPU: each computes its column shard and its epilogue writes
    the tiles into both ranks' row-major buffers through CUDA IPC mappings; both end with the
    full product, bit-identical to the unsharded GEMM."""
    import torch.multiprocessing as mp
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_ipc_worker, args=(r, 2, port, q)) for r in range(2)]
    for p in procs:
        p.start()
    res = [q.get(timeout=300) for _ in procs]
    for p in procs:
        p.join(timeout=60)
    assert all(ok for _, ok, _ in res), res
