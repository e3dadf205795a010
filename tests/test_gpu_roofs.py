"""GPU: the roofline probes and the bounded-wait failure path (no fault, no hang)."""
import pytest
import torch

pytestmark = pytest.mark.gpu


def test_bounded_wait_times_out_cleanly(api):
    word = api.wait_selftest(20_000_000)  # 20 ms limit on a barrier nothing completes
    assert word & (1 << 5)
    assert api.device_error() == 0       # cleared by the self test
    x = api.fill_uniform(4, 16, 1)       # the context is still usable
    torch.cuda.synchronize()
    assert x.abs().max().item() <= 1.0


def test_hbm_probe(api):
    n = 1 << 30
    a = torch.empty(n, dtype=torch.uint8, device="cuda")
    b = torch.empty(n, dtype=torch.uint8, device="cuda")
    gbs = api.measure_bandwidth(0, a, b, None, n, iters=5)
    assert 2000 < gbs < 9000
    gbs_r = api.measure_bandwidth(1, a, b, None, n, iters=5)
    assert 2000 < gbs_r < 9000


def test_peak_ladder(api):
    tf = api.peak(256, 148, 2048, 3)
    assert tf > 1000  # TFLOP/s; dense FP4 nominal is about 9000 at boost clock
    assert api.device_error() == 0


@pytest.mark.parametrize("cta_group", [1, 2])
def test_peak_ladder_random_data_and_clock(api, cta_group):
    units = 148 if cta_group == 1 else 74
    tf, mhz = api.peak_ex(256, cta_group, units, 2048, 3, seed=0x5EED)
    assert tf > 1000 and 300 < mhz < 2200
    tf_s, mhz_s = api.peak_ex(256, cta_group, units, 2048, 20, seed=0x5EED, sustained=True)
    assert tf_s > 1000 and 300 < mhz_s < 2200
    # Same issue rate per cycle whatever the data: TF/s per MHz agree within 15%.
    assert abs(tf / mhz - tf_s / mhz_s) / (tf / mhz) < 0.15
    with pytest.raises(api.Nvfp4Error):
        api.peak_ex(128, 2, units, 16, 1)
    assert api.device_error() == 0


def test_peak_ladder_sparse_rung(api):
    """The .sp rung counts 128 logical K per MMA: about twice the dense rung's FLOP rate."""
    dense, _ = api.peak_ex(128, 1, 148, 2048, 3, seed=0x5EED)
    sparse, _ = api.peak_ex(128, 1, 148, 2048, 3, seed=0x5EED, sparse=True)
    assert sparse > 1.3 * dense
    with pytest.raises(api.Nvfp4Error):
        api.peak_ex(256, 2, 74, 16, 1, sparse=True)
    assert api.device_error() == 0
