"""GPU: codecs byte-identical to the oracle (which is pinned to the reference's src/nvfp4.cu)."""
import os

import numpy as np
import pytest
import torch

pytestmark = pytest.mark.gpu
GOLD = os.path.join(os.path.dirname(os.path.abspath(__file__)), "golden")


def test_fill_uniform_bit_exact(api, orc):
    for rows, cols, seed in ((16, 256, 1234), (37, 96, 0), (256, 1024, 1234 ^ 0xABCDEF)):
        g = api.fill_uniform(rows, cols, seed).cpu().numpy()
        assert np.array_equal(g.view(np.uint32), orc.make_uniform(rows, cols, seed).view(np.uint32))


def test_fill_normal_moments(api):
    x = api.fill_normal(1024, 4096, 1234).double()
    assert abs(x.mean().item()) < 2e-3 and abs(x.std().item() - 1.0) < 2e-3
    y = api.fill_normal(1024, 4096, 1234)
    assert torch.equal(x.float(), y)  # deterministic


def test_quantize_golden_fixture(api):
    g = np.load(os.path.join(GOLD, "quant_small.npz"))
    for name in ("a", "b", "n"):
        x = torch.from_numpy(g[name]).cuda()
        t = api.quantize(x)
        assert np.array_equal(t.packed.cpu().numpy(), g[name + "_packed"]), name
        assert np.array_equal(t.scales.cpu().numpy(), g[name + "_scales"]), name
        dq = api.dequantize(t).cpu().numpy()
        assert np.array_equal(dq.view(np.uint32), g[name + "_dq"].view(np.uint32)), name
    t = api.quantize(torch.from_numpy(g["n"]).cuda(), 0.5)
    assert np.array_equal(t.packed.cpu().numpy(), g["n_g05_packed"])
    assert np.array_equal(t.scales.cpu().numpy(), g["n_g05_scales"])


@pytest.mark.parametrize("dist", ["normal", "uniform", "wide"])
def test_quantize_matches_oracle(api, orc, dist):
    rows, cols = 512, 2048
    if dist == "normal":
        x = api.fill_normal(rows, cols, 99)
    elif dist == "uniform":
        x = api.fill_uniform(rows, cols, 1234)
    else:  # scales across the whole UE4M3 range, subnormal scales and clamping included
        x = api.fill_normal(rows, cols, 5)
        x *= torch.exp(torch.linspace(-14, 9, rows, device="cuda")).unsqueeze(1)
        x[0, :16] = 0
        x[1, 3] = float("nan")
        x[2, 7] = float("inf")
        x[3, 9] = -float("inf")
    xh = x.cpu().numpy()
    for g in (1.0, 0.37):
        t = api.quantize(x, g)
        p, s = orc.quantize(xh, g)
        assert np.array_equal(t.packed.cpu().numpy(), p)
        assert np.array_equal(t.scales.cpu().numpy(), s)
        assert np.array_equal(t.scales_tc.cpu().numpy(), orc.sf_to_tcgen05(s, cols))
        dq = api.dequantize(t).cpu().numpy()
        assert np.array_equal(dq.view(np.uint32), orc.dequantize(p, s, cols, g).view(np.uint32))


def test_e4m3_boundaries(api, orc):
    """Scales at every midpoint between adjacent UE4M3 codes, +-8 ulps, through the quantiser."""
    L = orc.lib()
    dec = np.array([L.orc_e4m3_decode(c) for c in range(128)], np.float64)
    mids = ((dec[:-1] + dec[1:]) / 2).astype(np.float32)
    xs = np.concatenate([(np.float32(m).view(np.int32) + np.arange(-8, 9, dtype=np.int32)).view(np.float32)
                         for m in mids])
    xs = xs[xs > 0]
    # a block whose amax is 6*x has scale x (amax/6 is exact for these values? not always:
    # the quantiser's own division is part of what is compared).
    n = xs.size
    blocks = np.zeros((n, 16), np.float32)
    blocks[:, 0] = xs * np.float32(6.0)
    blocks[:, 1] = xs
    blocks[:, 2] = -xs * np.float32(2.5)
    t = api.quantize(torch.from_numpy(blocks).cuda())
    p, s = orc.quantize(blocks)
    assert np.array_equal(t.scales.cpu().numpy(), s)
    assert np.array_equal(t.packed.cpu().numpy(), p)


def test_sf_relayout_matches_oracle(api, orc):
    # Word-wide loads when K % 64 == 0 and the source is 4-byte aligned (1088: a partial second
    # tile of 16 atoms), byte loads otherwise (K = 16, 1040, and a source one byte off).
    for rows, K in ((128, 256), (300, 320), (1, 16), (1000, 4096), (129, 1088), (257, 1040)):
        s = torch.randint(0, 256, (rows, K // 16), dtype=torch.uint8, device="cuda")
        got = api.sf_to_tcgen05(s, rows, K).cpu().numpy()
        assert np.array_equal(got, orc.sf_to_tcgen05(s.cpu().numpy(), K))
    rows, K = 200, 512
    flat = torch.randint(0, 256, (rows * (K // 16) + 1,), dtype=torch.uint8, device="cuda")
    s = flat[1:].view(rows, K // 16)
    got = api.sf_to_tcgen05(s, rows, K).cpu().numpy()
    assert np.array_equal(got, orc.sf_to_tcgen05(s.cpu().numpy(), K))


def test_quantize_rejects_bad_shape(api):
    x = torch.zeros((4, 24), device="cuda")
    with pytest.raises(api.Nvfp4Error):
        api.quantize(x)


def test_e2m1_midpoints_and_huge_quotients(api, orc):
    """E2M1 rounding at every midpoint between adjacent magnitudes (+-4 ulps) with an exact
    unit scale (each block's amax is 6, so the divisor is 1), and blocks whose quotients pass
    2^25, where the reference's loop over rounded errors decides ties its own way (the scale
    clamps at 448, so x / 448 reaches that range)."""
    mids = np.array([0.25, 0.75, 1.25, 1.75, 2.5, 3.5, 5.0], np.float32)
    vals = np.concatenate([(m.view(np.int32) + np.arange(-4, 5, dtype=np.int32)).view(np.float32)
                           for m in mids])
    vals = np.concatenate([vals, -vals])
    nblk = -(-len(vals) // 15)
    x = np.zeros((nblk, 16), np.float32)
    x[:, 0] = 6.0
    flat = np.zeros(nblk * 15, np.float32)
    flat[:len(vals)] = vals
    x[:, 1:] = flat.reshape(nblk, 15)
    huge = np.float32(448.0) * np.array([2.0 ** 25, 2.0 ** 25 * 1.5, 2.0 ** 26, 2.0 ** 30, 3e37 / 448,
                                         2.0 ** 24, 2.0 ** 25 - 8, 1e6, 7.0, 0.0, 1.0, 2.0 ** 27,
                                         2.0 ** 25 + 64, 5e36 / 448, 1e30 / 448, 6.0], np.float32)
    x = np.concatenate([x, huge[None, :], -huge[None, :]])
    if len(x) % 2:
        x = np.concatenate([x, np.zeros((1, 16), np.float32)])
    x = x.reshape(-1, 32)
    xg = torch.from_numpy(x).cuda()
    t = api.quantize(xg, 1.0)
    p, s = orc.quantize(x, 1.0)
    assert np.array_equal(t.packed.cpu().numpy(), p)
    assert np.array_equal(t.scales.cpu().numpy(), s)
