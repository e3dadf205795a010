"""CPU: the oracle restatement against the reference's own codecs and its golden fixtures."""
import json
import os

import numpy as np
import pytest

GOLD = os.path.join(os.path.dirname(os.path.abspath(__file__)), "golden")


@pytest.fixture(scope="module")
def kat():
    with open(os.path.join(GOLD, "codec_kat.json")) as f:
        return json.load(f)


def test_e2m1_quantize_kat(orc, kat):
    for x, code in kat["e2m1_quantize"]:
        assert orc.lib().orc_e2m1_quantize(x) == code, x


def test_e4m3_encode_kat(orc, kat):
    for x, code in kat["e4m3_encode"]:
        assert orc.lib().orc_e4m3_encode(x) == code, x


def test_decode_tables(orc, kat):
    for c in range(256):
        assert orc.lib().orc_e4m3_decode(c) == kat["e4m3_decode"][c]
    for c in range(16):
        assert orc.lib().orc_e2m1_decode(c) == kat["e2m1_decode"][c]


def test_random_codec_kat(orc, kat):
    xs = np.array(kat["random_inputs_f32_hex"], np.uint32).view(np.float32)
    L = orc.lib()
    for x, e, s in zip(xs, kat["random_e2m1"], kat["random_e4m3"]):
        assert L.orc_e2m1_quantize(float(x)) == e
        assert L.orc_e4m3_encode(float(abs(x))) == s


def test_uniform_first_values(orc, kat):
    got = orc.make_uniform(1, 8, 1234)[0]
    assert [float(v) for v in got] == kat["uniform_seed1234_first8"]
    # splitmix64 first values for seed 1234 (src/nvfp4.cu:115-129)
    np.testing.assert_allclose(got[:4], [0.461333036, 0.185779691, -0.595734358, -0.387626529],
                               rtol=0, atol=1e-8)


def test_quantize_golden(orc):
    g = np.load(os.path.join(GOLD, "quant_small.npz"))
    for name in ("a", "b", "n"):
        p, s = orc.quantize(g[name])
        assert np.array_equal(p, g[name + "_packed"]), name
        assert np.array_equal(s, g[name + "_scales"]), name
        dq = orc.dequantize(p, s, g[name].shape[1])
        assert np.array_equal(dq, g[name + "_dq"]), name
    p, s = orc.quantize(g["n"], 0.5)
    assert np.array_equal(p, g["n_g05_packed"]) and np.array_equal(s, g["n_g05_scales"])
    assert np.array_equal(orc.make_uniform(16, 256, 1234), g["a"])
    assert np.array_equal(orc.make_uniform(16, 256, 1234 ^ 0xABCDEF), g["b"])


@pytest.mark.skipif(not os.path.exists(os.path.join(os.path.dirname(GOLD), "..", "oracle", "_ref",
                                                     "libnvfp4ref.so")),
                    reason="reference build absent")
def test_oracle_matches_reference_build_random(orc):
    rng = np.random.default_rng(3)
    x = (rng.standard_normal((64, 512)) * rng.uniform(1e-3, 50, (64, 1))).astype(np.float32)
    x[3, 10:20] = 0
    x[4, 0] = np.inf
    x[5, 0] = -np.inf
    x[6, 3] = np.nan
    for g in (1.0, 0.25, 3.0):
        p1, s1 = orc.quantize(x, g)
        p2, s2 = orc.quantize(x, g, use_ref=True)
        assert np.array_equal(p1, p2) and np.array_equal(s1, s2)
        d1 = orc.dequantize(p1, s1, 512, g)
        d2 = orc.dequantize(p1, s1, 512, g, use_ref=True)
        assert np.array_equal(d1.view(np.uint32), d2.view(np.uint32))


@pytest.mark.skipif(not os.path.exists(os.path.join(os.path.dirname(GOLD), "..", "oracle", "_ref",
                                                     "libnvfp4ref.so")),
                    reason="reference build absent")
def test_e4m3_encode_dense_sweep_vs_reference(orc):
    """Every float around every midpoint between adjacent scale codes, +-64 ulps."""
    L, R = orc.lib(), orc.ref()
    dec = np.array([L.orc_e4m3_decode(c) for c in range(128)], np.float32)
    mids = ((dec[:-1].astype(np.float64) + dec[1:]) / 2).astype(np.float32)
    xs = []
    for m in list(mids) + [np.float32(448.0)]:
        b = np.float32(m).view(np.int32)
        xs.append((b + np.arange(-64, 65, dtype=np.int32)).view(np.float32))
    xs = np.concatenate(xs)
    for x in xs[::3]:
        assert L.orc_e4m3_encode(float(x)) == R.ref_e4m3_encode(float(x)), float(x)


def test_int_gemm_kat(orc):
    """Exact-integer known answer of the reference's self-check (src/gemm_warp_mxf4.cu:124-157)."""
    g = np.load(os.path.join(GOLD, "int_gemm.npz"))
    mag = np.array([0, .5, 1, 1.5, 2, 3, 4, 6], np.float32)
    a = mag[g["codes_a"]]
    b_nk = mag[g["codes_b_kn"]].T.copy()
    c = orc.gemm_nt(a, b_nk)
    assert np.array_equal(c, g["c"])


def test_gemm_nt_matches_float64(orc):
    rng = np.random.default_rng(1)
    a = rng.standard_normal((33, 80)).astype(np.float32)
    b = rng.standard_normal((17, 80)).astype(np.float32)
    c = orc.gemm_nt(a, b, threads=3)
    ref = a.astype(np.float64) @ b.astype(np.float64).T
    assert np.abs(c - ref).max() < 1e-4
    rows = [0, 5, 32]
    assert np.array_equal(orc.gemm_nt_rows(a, b, rows, threads=2), c[rows])


def test_sf_tcgen05_layout(orc):
    rows, K = 300, 320
    s = np.arange(rows * K // 16, dtype=np.uint32).astype(np.uint8).reshape(rows, K // 16)
    t = orc.sf_to_tcgen05(s, K)
    assert t.size == 3 * 5 * 512
    ka = 5
    for r in (0, 1, 31, 32, 127, 128, 200, 299):
        for si in (0, 3, 4, 19):
            off = ((r // 128) * ka + si // 4) * 512 + (r % 32) * 16 + ((r // 32) % 4) * 4 + si % 4
            assert t[off] == s[r, si]
    # padding rows are zero
    assert t[(2 * ka) * 512 + 31 * 16 + 3 * 4] == 0  # row 2*128+3*32+31 = 383 >= 300


def test_sparse_meta_keeps_two_pairs(orc):
    """Pair-wise 2:4: every group of 8 keeps exactly 2 distinct pairs, first < second."""
    meta = orc.sparse_meta(8, 128, 0x24)
    nib = np.stack([meta & 0xF, meta >> 4], -1).reshape(8, 16)
    first, second = nib & 3, nib >> 2
    assert np.all(first < second)
    a = np.ones((8, 128), np.float32)
    z = orc.sparse_prune(a, meta)
    pairs = (z.reshape(8, 16, 4, 2) != 0)
    assert np.all(pairs.all(-1) == pairs.any(-1))          # pairs are kept or dropped whole
    assert np.all(pairs.all(-1).sum(-1) == 2)
    # all 6 combinations occur
    combos = set(zip(first.ravel().tolist(), second.ravel().tolist()))
    assert combos == {(0, 1), (0, 2), (0, 3), (1, 2), (1, 3), (2, 3)}


def test_quantize_block16_is_quantize(orc):
    x = orc.make_uniform(16, 256, 99) * 7
    p16, s16 = orc.quantize(x)
    pb, sb = orc.quantize_block(x, 16)
    assert np.array_equal(p16, pb) and np.array_equal(s16, sb)


def test_quantize_block32_semantics(orc):
    """Block 32: one scale per 32 elements, chosen exactly as for 16 (amax/6/g, e4m3 nearest)."""
    x = orc.make_uniform(4, 128, 5) * 3
    p32, s32 = orc.quantize_block(x, 32)
    assert s32.shape == (4, 4)
    for r in range(4):
        for b in range(4):
            amax = np.abs(x[r, 32 * b:32 * b + 32]).max()
            assert s32[r, b] == orc.lib().orc_e4m3_encode(float(np.float32(amax) / np.float32(6.0)))
    d = orc.dequantize_block(p32, s32, 128, 32)
    assert np.abs(d - x).max() <= np.abs(x).max() / 6 * 1.01  # within one e2m1 step of each scale


def test_sparse_compress_round_trip(orc):
    rows, K = 16, 256
    meta = orc.sparse_meta(rows, K, 7)
    x = orc.sparse_prune(orc.make_uniform(rows, K, 8), meta)
    packed, _ = orc.quantize_block(x, 32)
    vals = orc.sparse_compress(packed, meta, K)
    # Decompress by hand: put each kept pair byte back in its slot.
    back = np.zeros_like(packed)
    nib = np.stack([meta & 0xF, meta >> 4], -1).reshape(rows, K // 8)
    for r in range(rows):
        for g in range(K // 8):
            back[r, 4 * g + (nib[r, g] & 3)] = vals[r, 2 * g]
            back[r, 4 * g + (nib[r, g] >> 2)] = vals[r, 2 * g + 1]
    assert np.array_equal(back, packed)
