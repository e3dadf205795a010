"""GPU: the tcgen05 GEMM against the CPU oracle (src/reference.cu restated) through the C ABI.

Criterion (north_star): max |err| <= 1e-3 * max |C_ref| with FP32 output; BF16 output adds
half a BF16 ulp of |C_ref| for the final rounding.
"""
import os

import numpy as np
import pytest
import torch

from gpu_helpers import check_gemm, make_operand, oracle_dequant, run_gemm

pytestmark = pytest.mark.gpu
GOLD = os.path.join(os.path.dirname(os.path.abspath(__file__)), "golden")


def _case(api, orc, M, N, K, seed=11, dist="normal", out=torch.float32, ga=1.0, gb=1.0, **kw):
    _, a = make_operand(api, M, K, seed, dist, ga)
    _, b = make_operand(api, N, K, seed ^ 0xABCDEF, dist, gb)
    c = run_gemm(api, a, b, M, N, K, out_dtype=out, **kw)
    ref = orc.gemm_nt(oracle_dequant(orc, a), oracle_dequant(orc, b))
    return check_gemm(c.float().cpu().numpy(), ref, bf16=(out == torch.bfloat16))


def test_int_gemm_known_answer(api):
    """The reference's exact-integer self-check (src/gemm_warp_mxf4.cu:124-157): codes 0..7,
    unit scales (UE4M3 0x38 = 1.0); the answer is exact, so the error must be 0."""
    g = np.load(os.path.join(GOLD, "int_gemm.npz"))
    ca, cb = g["codes_a"], g["codes_b_kn"].T.copy()

    def pack(codes):
        return torch.from_numpy((codes[:, 0::2] | (codes[:, 1::2] << 4)).astype(np.uint8)).cuda()

    sc = torch.full((128, 8), 0x38, dtype=torch.uint8, device="cuda")
    out = torch.empty((128, 128), dtype=torch.float32, device="cuda")
    api.gemm(pack(ca), sc, pack(cb), sc, 128, 128, 128, out, sf_layout=api.SF_CANONICAL)
    torch.cuda.synchronize()
    assert np.array_equal(out.cpu().numpy(), g["c"])


def test_c1_1024_cubed_fp32(api, orc):
    """M=N=K=1024, N(0,1) operands, FP32 output."""
    _case(api, orc, 1024, 1024, 1024)


@pytest.mark.parametrize("tile_n", [128, 256])
def test_tiles_and_bf16(api, orc, tile_n):
    _case(api, orc, 512, 768, 1024, out=torch.bfloat16, tile_n=tile_n)
    _case(api, orc, 384, 512, 512, tile_n=tile_n)


@pytest.mark.parametrize("shape", [(128, 128, 64), (128, 256, 256), (200, 300, 320), (1, 16, 64),
                                   (129, 257, 288), (17, 1000, 96), (640, 200, 2048)])
def test_ragged_shapes(api, orc, shape):
    M, N, K = shape
    _case(api, orc, M, N, K, seed=M + N + K)


def test_canonical_layout_and_global_scales(api, orc):
    _case(api, orc, 256, 384, 512, sf_layout=api.SF_CANONICAL, ga=0.5, gb=3.0)
    _case(api, orc, 256, 384, 512, dist="uniform", ga=2.0, gb=0.25, out=torch.bfloat16)


def test_many_tiles_persistent(api, orc):
    """More tiles than SMs: the persistent loop, both accumulator buffers and their overlap."""
    _case(api, orc, 2048, 4096, 512, out=torch.bfloat16, tile_n=256)
    _case(api, orc, 2048, 2048, 512, tile_n=128)


def test_c2_shape_sampled_rows(api, orc):
    """BASELINE config 2 (4096 x 14336 x 4096, BF16 out): 96 sampled rows vs the oracle."""
    M, N, K = 4096, 14336, 4096
    _, a = make_operand(api, M, K, 1234)
    _, b = make_operand(api, N, K, 1234 ^ 0xABCDEF)
    c = run_gemm(api, a, b, M, N, K, out_dtype=torch.bfloat16)
    rows = np.unique(np.concatenate([np.arange(0, M, 97), [M - 1, 127, 128, 255]]))[:96]
    adq = oracle_dequant(orc, a)
    bdq = oracle_dequant(orc, b)
    ref = orc.gemm_nt_rows(adq, bdq, rows)
    check_gemm(c[torch.from_numpy(rows).long().cuda()].float().cpu().numpy(), ref, bf16=True)


def test_repeat_is_deterministic(api):
    M, N, K = 512, 1024, 1024
    _, a = make_operand(api, M, K, 3)
    _, b = make_operand(api, N, K, 4)
    c1 = run_gemm(api, a, b, M, N, K)
    c2 = run_gemm(api, a, b, M, N, K)
    assert torch.equal(c1, c2)


def test_rejects_bad_k(api):
    x = torch.zeros((128, 48), device="cuda")
    t = api.quantize(x)
    out = torch.empty((128, 128), device="cuda")
    with pytest.raises(api.Nvfp4Error):
        api.gemm(t.packed, t.scales, t.packed, t.scales, 128, 128, 48, out,
                 sf_layout=api.SF_CANONICAL)


@pytest.mark.parametrize("shape", [(256, 256, 256), (512, 768, 1024), (300, 520, 288), (100, 256, 64),
                                   (1000, 1000, 2048), (2048, 4096, 512)])
@pytest.mark.parametrize("out", [torch.float32, torch.bfloat16])
def test_sm_pair_kernel(api, orc, shape, out):
    """The cta_group::2 kernel (256 x 256 tiles on SM pairs), forced, on ragged shapes."""
    M, N, K = shape
    _case(api, orc, M, N, K, seed=M * 7 + N + K, out=out, cta_group=2)


def test_sm_pair_matches_one_sm(api):
    """Both kernels accumulate in FP32 per K-block in the same order: identical outputs."""
    M, N, K = 1024, 2048, 1024
    _, a = make_operand(api, M, K, 21)
    _, b = make_operand(api, N, K, 22)
    c1 = run_gemm(api, a, b, M, N, K, cta_group=1, tile_n=256)
    c2 = run_gemm(api, a, b, M, N, K, cta_group=2)
    assert torch.equal(c1, c2)


@pytest.mark.parametrize("shape", [(16, 14336, 4096), (64, 4096, 14336), (128, 1024, 2048),
                                   (1, 300, 512), (17, 1000, 96), (100, 2000, 4096),
                                   (33, 256, 8192), (32, 4096, 14336), (8, 2048, 4096),
                                   (16, 4096, 14336), (128, 4096, 14336), (128, 14336, 4096),
                                   (5, 128, 1088), (64, 640, 320)])
@pytest.mark.parametrize("out", [torch.float32, torch.bfloat16])
def test_decode_kernel(api, orc, shape, out):
    """M <= 128 (the weight-streaming split-K kernel where the heuristic picks it, else the
    general kernel)."""
    M, N, K = shape
    _case(api, orc, M, N, K, seed=M + 3 * N + K, out=out)


def test_decode_repeat_deterministic(api):
    """Split-K partial sums are reduced in cluster-rank order through distributed shared
    memory: repeated calls agree bit for bit, and the BF16 output is the rounded FP32 one."""
    M, N, K = 16, 4096, 14336
    _, a = make_operand(api, M, K, 41)
    _, b = make_operand(api, N, K, 42)
    c1 = run_gemm(api, a, b, M, N, K)
    c2 = run_gemm(api, a, b, M, N, K)
    c3 = run_gemm(api, a, b, M, N, K, out_dtype=torch.bfloat16)
    assert torch.equal(c1, c2)
    assert torch.equal(c1.to(torch.bfloat16), c3)


def test_decode_matches_general_kernel(api):
    M, N, K = 64, 2048, 4096
    _, a = make_operand(api, M, K, 51)
    _, b = make_operand(api, N, K, 52)
    d = run_gemm(api, a, b, M, N, K)
    g = run_gemm(api, a, b, M, N, K, cta_group=1, tile_n=128)
    scale = g.abs().max().item()
    assert (d - g).abs().max().item() <= 1e-5 * scale


@pytest.mark.parametrize("cta_group", [1, 2])
def test_fresh_operand_buffers_reproduce(api, cta_group):
    """Regression: launches on freshly written operand copies (slow first-touch loads) must
    reproduce the first result bit for bit. This caught a scale-writer race in which one
    writer group consumed a stage's scales before the bytes had landed."""
    M, N, K = 4096, 14336, 4096
    _, a = make_operand(api, M, K, 1234)
    _, b = make_operand(api, N, K, 1234 ^ 0xABCDEF)
    ref = run_gemm(api, a, b, M, N, K, out_dtype=torch.bfloat16, cta_group=cta_group, tile_n=256)
    for _ in range(6):
        a2 = api.Nvfp4Tensor(a.rows, a.cols, a.global_scale, a.packed.clone(), a.scales.clone(),
                             a.scales_tc.clone())
        b2 = api.Nvfp4Tensor(b.rows, b.cols, b.global_scale, b.packed.clone(), b.scales.clone(),
                             b.scales_tc.clone())
        got = run_gemm(api, a2, b2, M, N, K, out_dtype=torch.bfloat16, cta_group=cta_group,
                       tile_n=256)
        assert torch.equal(got, ref)
        del a2, b2


@pytest.mark.parametrize("shape", [(16, 4096, 14336), (64, 14336, 4096), (100, 2000, 1024)])
def test_decode_b_static_is_identical(api, shape):
    """b_static only lets the decode kernel read the weight before the preceding kernel ends;
    the result must not change (here the preceding kernel quantises A on the same stream)."""
    M, N, K = shape
    x, a = make_operand(api, M, K, 71)
    _, b = make_operand(api, N, K, 72)
    ref = run_gemm(api, a, b, M, N, K)
    out = torch.empty((M, N), dtype=torch.float32, device="cuda")
    g = api.gemm_args(a.packed, a.scales_tc, b.packed, b.scales_tc, M, N, K, out, b_static=True)
    for _ in range(3):
        api.quantize(x, a.global_scale)          # re-quantise A just before the GEMM
        a2 = api.quantize(x, a.global_scale)
        g = api.gemm_args(a2.packed, a2.scales_tc, b.packed, b.scales_tc, M, N, K, out, b_static=True)
        api.launch(g)
        torch.cuda.synchronize()
        assert api.device_error() == 0
        assert torch.equal(out, ref)


def _dequant_rows(orc, t, rows):
    """Dequantise only the given rows of a GPU-quantised operand (canonical scales)."""
    idx = torch.from_numpy(np.asarray(rows)).long().cuda()
    p = t.packed[idx].cpu().numpy()
    s = t.scales[idx].cpu().numpy()
    return orc.dequantize(p, s, t.cols, t.global_scale)


def _tile_rows(M, extra=()):
    """One row in every 128-row tile row (a different offset in each), plus the given rows."""
    r = [t * 128 + (t * 37 + 5) % 128 for t in range((M + 127) // 128)]
    return np.unique(np.concatenate([np.array(r), np.array(extra, dtype=np.int64)])).astype(np.int32)


@pytest.mark.parametrize("cta_group", [0, 2])
def test_c3_8192_cubed_sampled_rows(api, orc, cta_group):
    """BASELINE config 3 on one GPU (8192^3, BF16 out): a row in every 128-row tile row (so
    every tile row of the persistent schedule and both accumulator buffers are sampled) plus
    the matrix edges, over all 8192 columns, against the oracle."""
    M = N = K = 8192
    _, a = make_operand(api, M, K, 1234)
    _, b = make_operand(api, N, K, 1234 ^ 0xABCDEF)
    c = run_gemm(api, a, b, M, N, K, out_dtype=torch.bfloat16, cta_group=cta_group)
    rows = _tile_rows(M, extra=(0, 127, 128, 255, 256, M - 1))
    assert len(rows) >= 64
    ref = orc.gemm_nt_rows(_dequant_rows(orc, a, rows), oracle_dequant(orc, b),
                           np.arange(len(rows), dtype=np.int32))
    check_gemm(c[torch.from_numpy(rows).long().cuda()].float().cpu().numpy(), ref, bf16=True)


def test_c3_16k_shard_sampled_rows(api, orc):
    """One GPU's shard of BASELINE config 3's large case over 8 GPUs: 16384 x (65536/8) x
    16384, BF16 out; a row in every 128-row tile row, all 8192 columns, against the oracle."""
    M, N, K = 16384, 65536 // 8, 16384
    _, a = make_operand(api, M, K, 1234)
    _, b = make_operand(api, N, K, (1234 ^ 0xABCDEF) + 3)
    c = run_gemm(api, a, b, M, N, K, out_dtype=torch.bfloat16)
    rows = _tile_rows(M, extra=(0, M - 1))
    assert len(rows) >= 128
    ref = orc.gemm_nt_rows(_dequant_rows(orc, a, rows), oracle_dequant(orc, b),
                           np.arange(len(rows), dtype=np.int32))
    check_gemm(c[torch.from_numpy(rows).long().cuda()].float().cpu().numpy(), ref, bf16=True)


@pytest.mark.parametrize("out", [torch.float32, torch.bfloat16])
def test_decode_up_proj_m64(api, orc, out):
    """BASELINE config 5, up-proj at M = 64 (64 x 14336 x 4096), every output against the
    oracle."""
    _case(api, orc, 64, 14336, 4096, seed=64 + 3 * 14336 + 4096, out=out)


@pytest.mark.parametrize("shape", [(16, 4096, 14336), (64, 14336, 4096)])
def test_decode_b_static_with_canonical_scales(api, shape):
    """With canonical scales the call reorders B's scales itself just before the decode kernel,
    so B_STATIC must not let the kernel read them early: the output equals the one without
    the flag, on repeated calls whose reorder rewrites the workspace each time."""
    M, N, K = shape
    x, a = make_operand(api, M, K, 81)
    _, b = make_operand(api, N, K, 82)
    _, b2 = make_operand(api, N, K, 83)
    refs = [run_gemm(api, a, bb, M, N, K, sf_layout=api.SF_CANONICAL) for bb in (b, b2)]
    out = torch.empty((M, N), dtype=torch.float32, device="cuda")
    for i in range(4):
        bb = (b, b2)[i % 2]
        g = api.gemm_args(a.packed, a.scales, bb.packed, bb.scales, M, N, K, out,
                          sf_layout=api.SF_CANONICAL, b_static=True)
        api.launch(g)
        torch.cuda.synchronize()
        assert api.device_error() == 0
        assert torch.equal(out, refs[i % 2])


def test_canonical_calls_on_two_streams(api):
    """Canonical-scale calls on two streams at once: each stream reorders into its own
    workspace, so both results equal the serial ones."""
    shapes = [(512, 1024, 2048), (384, 768, 1024)]
    ops, refs = [], []
    for i, (M, N, K) in enumerate(shapes):
        _, a = make_operand(api, M, K, 90 + i)
        _, b = make_operand(api, N, K, 95 + i)
        ops.append((a, b, M, N, K))
        refs.append(run_gemm(api, a, b, M, N, K, sf_layout=api.SF_CANONICAL))
    streams = [torch.cuda.Stream(), torch.cuda.Stream()]
    outs = [torch.empty((M, N), dtype=torch.float32, device="cuda") for _, _, M, N, _ in ops]
    torch.cuda.synchronize()
    for _ in range(3):
        for (a, b, M, N, K), s, o in zip(ops, streams, outs):
            with torch.cuda.stream(s):
                api.gemm(a.packed, a.scales, b.packed, b.scales, M, N, K, o,
                         sf_layout=api.SF_CANONICAL, stream=s)
        torch.cuda.synchronize()
        assert api.device_error() == 0
        for o, r in zip(outs, refs):
            assert torch.equal(o, r)
