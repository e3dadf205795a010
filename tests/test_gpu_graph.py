"""GPU: the GEMM launched from a captured CUDA graph.

A serving loop captures its decode step once and replays it; the engine's launches must be
capturable (no allocation, no synchronisation, no host read-back inside a call) and a replay
must give the same bytes as the eager call. Covered: the regular entry point with tcgen05
scales on a decode shape (weight-streaming kernel, programmatic dependent launch between the
captured launches), a general shape (one-SM kernel) and a sparse shape, and the
allocation-free entry point with canonical scales (its scale reorder runs inside the graph).
"""
import ctypes as C

import pytest
import torch

from gpu_helpers import make_operand

pytestmark = pytest.mark.gpu


def _capture(fn, reps=3):
    """Capture `reps` calls of fn() into a graph; return the graph (not yet replayed)."""
    g = torch.cuda.CUDAGraph()
    s = torch.cuda.Stream()
    s.wait_stream(torch.cuda.current_stream())
    with torch.cuda.stream(s):
        with torch.cuda.graph(g, stream=s):
            for _ in range(reps):
                fn()
    torch.cuda.current_stream().wait_stream(s)
    return g


@pytest.mark.parametrize("M,N,K", [(16, 1024, 2048), (128, 4096, 512), (512, 768, 1024)])
def test_graph_replay_matches_eager(api, M, N, K):
    _, a = make_operand(api, M, K, 31, global_scale=0.5)
    _, b = make_operand(api, N, K, 32, global_scale=2.0)
    ref = torch.empty((M, N), dtype=torch.bfloat16, device="cuda")
    out = torch.full((M, N), float("nan"), dtype=torch.bfloat16, device="cuda")
    eager = api.gemm_args(a.packed, a.scales_tc, b.packed, b.scales_tc, M, N, K, ref,
                          a_global=a.global_scale, b_global=b.global_scale, sf_layout=api.SF_TCGEN05)
    cap = api.gemm_args(a.packed, a.scales_tc, b.packed, b.scales_tc, M, N, K, out,
                        a_global=a.global_scale, b_global=b.global_scale, sf_layout=api.SF_TCGEN05)
    api.launch(eager)
    api.launch(cap)  # first call on this shape outside the capture (attributes, tensor maps)
    torch.cuda.synchronize()
    out.fill_(float("nan"))
    torch.cuda.synchronize()
    g = _capture(lambda: api.launch(cap))
    g.replay()
    g.replay()
    torch.cuda.synchronize()
    assert api.device_error() == 0
    assert torch.equal(out, ref)


def test_graph_replay_sparse(api):
    M, N, K = 256, 512, 1024
    x = api.fill_normal(M, K, 41)
    meta = api.sparse_meta(M, K, 0x24)
    api.sparse_prune(x, meta)
    ta = api.quantize_block(x, 32)
    vals = api.sparse_compress(ta.packed, meta, K)
    tb = api.quantize_block(api.fill_normal(N, K, 42), 32)
    ref = torch.empty((M, N), dtype=torch.bfloat16, device="cuda")
    out = torch.empty((M, N), dtype=torch.bfloat16, device="cuda")
    mk = lambda c: api.gemm_args(vals, ta.scales_tc, tb.packed, tb.scales_tc, M, N, K, c,
                                 sf_layout=api.SF_TCGEN05, mode=api.MODE_SPARSE24, a_meta=meta)
    args_ref, args = mk(ref), mk(out)
    api.launch(args_ref)
    api.launch(args)
    torch.cuda.synchronize()
    out.zero_()
    g = _capture(lambda: api.launch(args))
    g.replay()
    torch.cuda.synchronize()
    assert api.device_error() == 0
    assert torch.equal(out, ref)


def test_graph_noalloc_canonical_scales(api):
    """The allocation-free entry point reorders canonical scales inside the captured graph."""
    L = api.lib()
    M, N, K = 64, 768, 1024
    _, a = make_operand(api, M, K, 51, global_scale=0.5)
    _, b = make_operand(api, N, K, 52, global_scale=2.0)
    ref = torch.empty((M, N), dtype=torch.bfloat16, device="cuda")
    out = torch.full((M, N), float("nan"), dtype=torch.bfloat16, device="cuda")

    def args_for(c):
        return api.GemmArgs(a.packed.data_ptr(), a.scales.data_ptr(), a.global_scale,
                            b.packed.data_ptr(), b.scales.data_ptr(), b.global_scale,
                            c.data_ptr(), M, N, K, api.MODE_DENSE, api.SF_CANONICAL,
                            api.OUT_BF16, None, 0, 0)

    err = C.create_string_buffer(512)
    rc = L.nvfp4_b200_gemm(C.byref(args_for(ref)), C.c_void_p(torch.cuda.current_stream().cuda_stream),
                           err, 512)
    assert rc == 0, err.value.decode()
    cargs = args_for(out)
    rcs = []

    def call():
        rcs.append(L.nvfp4_b200_gemm_noalloc(C.byref(cargs),
                                             C.c_void_p(torch.cuda.current_stream().cuda_stream),
                                             err, 512))

    call()  # eager once (attributes, tensor maps)
    torch.cuda.synchronize()
    out.fill_(float("nan"))
    torch.cuda.synchronize()
    rcs.clear()
    g = _capture(call, reps=2)
    assert rcs == [0, 0], err.value.decode()
    g.replay()
    torch.cuda.synchronize()
    assert api.device_error() == 0
    assert torch.equal(out, ref)
