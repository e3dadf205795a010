"""The division-free E2M1 rule of the GPU quantiser (codec_dev.cuh, e2m1_thresholds /
e2m1_code_fast), restated in numpy and checked against the reference's form: the count of
midpoints {.25,.75,1.25,1.75,2.5,3.5,5} strictly below fl(|x| / dec) (src/nvfp4.cu:18-29, 88-92),
with the sign bit of the rounded quotient. CPU only; the GPU tests check the kernel's bytes."""
import numpy as np

MIDS = np.array([0.25, 0.75, 1.25, 1.75, 2.5, 3.5, 5.0])
# m + ulp(m)/2 for each midpoint (float32 ulp)
BOUNDS = MIDS + np.array([2.0 ** -26, 2.0 ** -25, 2.0 ** -24, 2.0 ** -24, 2.0 ** -23, 2.0 ** -23,
                          2.0 ** -22])


def _round_down_f32(v):
    f = v.astype(np.float32)
    return np.where(f.astype(np.float64) > v, np.nextafter(f, np.float32(-np.inf)), f)


def _round_up_f32(v):
    f = v.astype(np.float32)
    return np.where(f.astype(np.float64) < v, np.nextafter(f, np.float32(np.inf)), f)


def _by_division(x, dec):
    q = (x / dec).astype(np.float32)  # IEEE single division, rounded to nearest even
    a = np.abs(q)
    code = (a[:, None] > MIDS[None, :].astype(np.float32)).sum(axis=1)
    return code | np.where(q < 0, 8, 0)


def _by_thresholds(x, dec):
    d = dec.astype(np.float64)
    t = _round_down_f32(BOUNDS[None, :] * d[:, None])
    zero = _round_down_f32(2.0 ** -150 * d)
    a = np.abs(x)
    code = (a[:, None] > t).sum(axis=1)
    return code | np.where((x < 0) & (a > zero), 8, 0), a < _round_up_f32(16777216.0 * d)


def _check(x, dec):
    with np.errstate(over="ignore", under="ignore", invalid="ignore", divide="ignore"):
        want = _by_division(x, dec)
        got, fast = _by_thresholds(x, dec)
    assert fast.any()
    bad = fast & (want != got)
    assert not bad.any(), (x[bad][:5], dec[bad][:5], want[bad][:5], got[bad][:5])


def test_rule_random_bits():
    rng = np.random.default_rng(7)
    x = rng.integers(0, 2 ** 32, 2_000_000, dtype=np.uint64).astype(np.uint32).view(np.float32)
    dec = np.abs(rng.integers(0, 2 ** 32, 2_000_000, dtype=np.uint64).astype(np.uint32)
                 .view(np.float32))
    ok = np.isfinite(dec) & (dec > 0) & ~np.isnan(x)
    _check(x[ok], dec[ok])


def test_rule_at_midpoints():
    """|x| within a few ulps of midpoint * dec, the cases where the division's rounding decides."""
    rng = np.random.default_rng(11)
    n = 2_000_000
    dec = np.abs(rng.standard_normal(n).astype(np.float32) * np.float32(2.0) **
                 rng.integers(-40, 40, n).astype(np.float32)).astype(np.float32)
    dec = dec[dec > 0]
    m = MIDS[rng.integers(0, 7, dec.size)]
    c = (m * dec.astype(np.float64)).astype(np.float32)
    bits = c.view(np.uint32).astype(np.int64) + rng.integers(-4, 5, dec.size)
    x = bits.astype(np.uint32).view(np.float32)
    x = np.where(rng.integers(0, 2, dec.size) == 1, -x, x).astype(np.float32)
    _check(x, dec)
