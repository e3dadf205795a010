"""GPU: activation quantisation fused into the GEMM (nvfp4_b200_gemm_quantize_a) through the C
ABI. Its A outputs must be byte-identical to the standalone quantiser (which is itself
byte-identical to the reference's quantize_to_nvfp4) and its C bit-identical to quantise +
nvfp4_b200_gemm on the same bytes, on consecutive calls (the fused kernel's grid barrier must
reset itself) with and without B_STATIC, on decode shapes (one fused launch) and on shapes that
take the two-launch path."""
import pytest
import torch

from gpu_helpers import make_operand

pytestmark = pytest.mark.gpu

# Fused single launch: M <= 128, K % 64 == 0 and N >= 74 128-row tiles (no K split): the up-proj
# shapes and the two wide ones; the rest take the quantiser + GEMM path.
SHAPES = [(16, 14336, 4096), (64, 14336, 4096), (128, 14336, 1088), (100, 10240, 1024),
          (1, 9600, 512), (16, 4096, 14336), (1, 256, 512), (100, 2000, 1024), (128, 1024, 2048),
          (256, 512, 1024), (16, 512, 96)]


@pytest.mark.parametrize("shape", SHAPES)
@pytest.mark.parametrize("b_static", [False, True])
def test_fused_quantize_matches_separate(api, shape, b_static):
    M, N, K = shape
    _, b = make_operand(api, N, K, 7)
    for rep, g in enumerate((1.0, 0.37)):
        x = api.fill_normal(M, K, 100 + rep)
        ref_a = api.quantize(x, g, canonical=False, tcgen05=True)
        ref = torch.empty((M, N), dtype=torch.bfloat16, device="cuda")
        api.gemm(ref_a.packed, ref_a.scales_tc, b.packed, b.scales_tc, M, N, K, ref,
                 a_global=g, sf_layout=api.SF_TCGEN05)
        pk = torch.full_like(ref_a.packed, 0xAB)
        sc = torch.full_like(ref_a.scales_tc, 0xCD)
        out = torch.full((M, N), float("nan"), dtype=torch.bfloat16, device="cuda")
        args = api.gemm_args(pk, sc, b.packed, b.scales_tc, M, N, K, out, a_global=g,
                             sf_layout=api.SF_TCGEN05, b_static=b_static)
        api.launch_quantize_a(args, x)
        torch.cuda.synchronize()
        assert api.device_error() == 0
        assert torch.equal(pk, ref_a.packed), "packed A differs from the standalone quantiser"
        assert torch.equal(sc, ref_a.scales_tc), "A scales differ from the standalone quantiser"
        assert torch.equal(out, ref), f"{shape} call {rep}: C differs from quantise + GEMM"


def test_fused_quantize_rejects_canonical_scales(api):
    M, N, K = 16, 256, 512
    x = api.fill_normal(M, K, 1)
    a = api.quantize(x)
    _, b = make_operand(api, N, K, 2)
    out = torch.empty((M, N), dtype=torch.float32, device="cuda")
    args = api.gemm_args(a.packed, a.scales, b.packed, b.scales, M, N, K, out,
                         sf_layout=api.SF_CANONICAL)
    with pytest.raises(api.Nvfp4Error):
        api.launch_quantize_a(args, x)
