"""GPU: pair-wise 2:4 sparse NVFP4 (GemmMode::Sparse).

The tcgen05 .sp kind::mxf4nvf4 MMA keeps 2 of the 4 element pairs of every group of 8 K
elements and applies one UE4M3 scale per 32 K elements of A and of B. The codecs (metadata,
prune, block-32 quantise, compress) are compared byte for byte with the CPU oracle, the GEMM
with the oracle's FP32 GEMM of the dequantised operands (max |err| <= 1e-3 * max |C|), and at
the C4 size with the dense kernel on the same math (decompressed A, each block-32 scale used for
both of its 16-element halves) plus sampled oracle rows.
"""
import numpy as np
import pytest
import torch

from gpu_helpers import check_gemm

pytestmark = pytest.mark.gpu

PATTERN_SEED = 0x24


def make_sparse_a(api, M, K, seed, pseed=PATTERN_SEED):
    x = api.fill_normal(M, K, seed)
    meta = api.sparse_meta(M, K, pseed)
    api.sparse_prune(x, meta)
    t = api.quantize_block(x, 32)
    vals = api.sparse_compress(t.packed, meta, K)
    return x, meta, t, vals


def sparse_gemm(api, vals, meta, ta, tb, M, N, K, out_dtype=torch.float32, canonical=False):
    out = torch.empty((M, N), dtype=out_dtype, device="cuda")
    sa, sb = (ta.scales, tb.scales) if canonical else (ta.scales_tc, tb.scales_tc)
    api.gemm(vals, sa, tb.packed, sb, M, N, K, out, mode=api.MODE_SPARSE24, a_meta=meta,
             sf_layout=api.SF_CANONICAL if canonical else api.SF_TCGEN05)
    torch.cuda.synchronize()
    assert api.device_error() == 0
    return out


def test_sparse_codecs_bit_exact(api, orc):
    M, K = 300, 640
    x, meta, t, vals = make_sparse_a(api, M, K, 11)
    torch.cuda.synchronize()
    m_ref = orc.sparse_meta(M, K, PATTERN_SEED)
    assert np.array_equal(meta.cpu().numpy(), m_ref)
    x0 = api.fill_normal(M, K, 11).cpu().numpy()
    xp_ref = orc.sparse_prune(x0, m_ref)
    assert np.array_equal(x.cpu().numpy().view(np.uint32), xp_ref.view(np.uint32))
    p_ref, s_ref = orc.quantize_block(xp_ref, 32)
    assert np.array_equal(t.packed.cpu().numpy(), p_ref)
    assert np.array_equal(t.scales.cpu().numpy(), s_ref)
    assert np.array_equal(t.scales_tc.cpu().numpy(), orc.sf_to_tcgen05(s_ref, K // 2))
    assert np.array_equal(vals.cpu().numpy(), orc.sparse_compress(p_ref, m_ref, K))
    d = api.dequantize_block(t, 32).cpu().numpy()
    assert np.array_equal(d.view(np.uint32), orc.dequantize_block(p_ref, s_ref, K, 32).view(np.uint32))


@pytest.mark.parametrize("shape", [(128, 128, 128), (128, 128, 512), (256, 384, 1024), (200, 300, 640),
                                   (1, 16, 128), (300, 520, 2048), (1000, 136, 384)])
@pytest.mark.parametrize("out", [torch.float32, torch.bfloat16])
def test_sparse_gemm_vs_oracle(api, orc, shape, out):
    M, N, K = shape
    _, meta, ta, vals = make_sparse_a(api, M, K, M + K)
    tb = api.quantize_block(api.fill_normal(N, K, N + 7), 32)
    c = sparse_gemm(api, vals, meta, ta, tb, M, N, K, out)
    A = orc.dequantize_block(ta.packed.cpu().numpy(), ta.scales.cpu().numpy(), K, 32)
    B = orc.dequantize_block(tb.packed.cpu().numpy(), tb.scales.cpu().numpy(), K, 32)
    check_gemm(c.float().cpu().numpy(), orc.gemm_nt(A, B), bf16=out == torch.bfloat16)


def test_sparse_gemm_canonical_scales(api, orc):
    M, N, K = 256, 256, 1024
    _, meta, ta, vals = make_sparse_a(api, M, K, 5)
    tb = api.quantize_block(api.fill_normal(N, K, 6), 32)
    c1 = sparse_gemm(api, vals, meta, ta, tb, M, N, K)
    c2 = sparse_gemm(api, vals, meta, ta, tb, M, N, K, canonical=True)
    assert torch.equal(c1, c2)


def test_sparse_mode_rejects_bad_arguments(api):
    M, N, K = 128, 128, 192   # K not a multiple of 128
    vals = torch.zeros((M, K // 4), dtype=torch.uint8, device="cuda")
    meta = torch.zeros((M, K // 16), dtype=torch.uint8, device="cuda")
    sc = torch.zeros(4096, dtype=torch.uint8, device="cuda")
    b = torch.zeros((N, K // 2), dtype=torch.uint8, device="cuda")
    out = torch.empty((M, N), dtype=torch.float32, device="cuda")
    with pytest.raises(api.Nvfp4Error):
        api.gemm(vals, sc, b, sc, M, N, K, out, mode=api.MODE_SPARSE24, a_meta=meta)
    with pytest.raises(api.Nvfp4Error):   # metadata missing
        api.gemm(vals, sc, b, sc, M, N, 256, out, mode=api.MODE_SPARSE24)


def test_sparse_c4_matches_dense_on_decompressed(api, orc):
    """C4 (4096 x 14336 x 8192): the sparse kernel against the dense kernel on the same math,
    and sampled rows against the oracle."""
    M, N, K = 4096, 14336, 8192
    x, meta, ta, vals = make_sparse_a(api, M, K, 1234)
    del x
    xb = api.fill_normal(N, K, 1234 ^ 0xABCDEF)
    tb = api.quantize_block(xb, 32)
    del xb
    cs = sparse_gemm(api, vals, meta, ta, tb, M, N, K)
    sa16 = ta.scales.repeat_interleave(2, dim=1).contiguous()
    sb16 = tb.scales.repeat_interleave(2, dim=1).contiguous()
    cd = torch.empty_like(cs)
    api.gemm(ta.packed, sa16, tb.packed, sb16, M, N, K, cd, sf_layout=api.SF_CANONICAL,
             cta_group=1, tile_n=256)
    torch.cuda.synchronize()
    scale = cd.abs().max().item()
    assert (cs - cd).abs().max().item() <= 1e-4 * scale
    rows = [0, 1, 777, 2048, 4095]
    A = orc.dequantize_block(ta.packed[rows].cpu().numpy(), ta.scales[rows].cpu().numpy(), K, 32)
    B = orc.dequantize_block(tb.packed.cpu().numpy(), tb.scales.cpu().numpy(), K, 32)
    check_gemm(cs[rows].cpu().numpy(), orc.gemm_nt(A, B))
