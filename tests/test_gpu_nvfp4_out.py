"""GPU: NVFP4 output epilogue (the GEMM writes C as packed E2M1 + UE4M3 scales, the next
layer's A operand). It must be byte-identical to quantising the same kernel's FP32 output
with the GPU codec (itself byte-identical to quantize_to_nvfp4, src/nvfp4.cu:62-97)."""
import pytest
import torch

from gpu_helpers import make_operand, run_gemm

pytestmark = pytest.mark.gpu


def nvfp4_out(api, a, b, M, N, K, layout, g, **kw):
    pk = torch.empty((M, N // 2), dtype=torch.uint8, device="cuda")
    if layout == api.SF_CANONICAL:
        sc = torch.empty((M, N // 16), dtype=torch.uint8, device="cuda")
    else:
        sc = torch.full((api.sf_tcgen05_bytes(M, N),), 0xAB, dtype=torch.uint8, device="cuda")
    api.gemm(a.packed, a.scales_tc, b.packed, b.scales_tc, M, N, K, pk, out_scales=sc,
             out_global=g, out_sf_layout=layout, **kw)
    torch.cuda.synchronize()
    assert api.device_error() == 0
    return pk, sc


@pytest.mark.parametrize("shape,kw", [
    ((256, 512, 1024), {}),
    ((300, 640, 320), {}),
    ((512, 1024, 512), dict(cta_group=1, tile_n=128)),
    ((512, 1024, 512), dict(cta_group=1, tile_n=256)),
    ((512, 512, 512), dict(cta_group=2)),
    ((64, 2048, 1024), dict(cta_group=1)),
])
@pytest.mark.parametrize("layout", ["canonical", "tcgen05"])
def test_nvfp4_output_matches_quantised_f32(api, shape, kw, layout):
    M, N, K = shape
    _, a = make_operand(api, M, K, 3)
    _, b = make_operand(api, N, K, 4)
    c32 = run_gemm(api, a, b, M, N, K, **kw)
    g = 0.25
    ref = api.quantize(c32, g)
    lay = api.SF_CANONICAL if layout == "canonical" else api.SF_TCGEN05
    pk, sc = nvfp4_out(api, a, b, M, N, K, lay, g, **kw)
    assert torch.equal(pk, ref.packed)
    assert torch.equal(sc, ref.scales if layout == "canonical" else ref.scales_tc)


def test_nvfp4_output_sparse_kernel(api):
    M, N, K = 256, 384, 1024
    x = api.fill_normal(M, K, 9)
    meta = api.sparse_meta(M, K, 0x24)
    api.sparse_prune(x, meta)
    ta = api.quantize_block(x, 32)
    vals = api.sparse_compress(ta.packed, meta, K)
    tb = api.quantize_block(api.fill_normal(N, K, 10), 32)
    c32 = torch.empty((M, N), dtype=torch.float32, device="cuda")
    api.gemm(vals, ta.scales_tc, tb.packed, tb.scales_tc, M, N, K, c32, mode=api.MODE_SPARSE24,
             a_meta=meta)
    pk = torch.empty((M, N // 2), dtype=torch.uint8, device="cuda")
    sc = torch.empty((M, N // 16), dtype=torch.uint8, device="cuda")
    api.gemm(vals, ta.scales_tc, tb.packed, tb.scales_tc, M, N, K, pk, mode=api.MODE_SPARSE24,
             a_meta=meta, out_scales=sc, out_global=1.0)
    torch.cuda.synchronize()
    ref = api.quantize(c32, 1.0)
    assert torch.equal(pk, ref.packed) and torch.equal(sc, ref.scales)


def test_nvfp4_output_rejects_ragged_n(api):
    M, N, K = 128, 48, 256     # N not a multiple of 32
    _, a = make_operand(api, M, K, 1)
    _, b = make_operand(api, N, K, 2)
    pk = torch.empty((M, N // 2), dtype=torch.uint8, device="cuda")
    sc = torch.empty((M, N // 16), dtype=torch.uint8, device="cuda")
    with pytest.raises(api.Nvfp4Error):
        api.gemm(a.packed, a.scales_tc, b.packed, b.scales_tc, M, N, K, pk, out_scales=sc,
                 cta_group=1)
