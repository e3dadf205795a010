"""CPU: bench.py's host-side logic (configs, algorithmic bytes, sharding of the configs)."""
import os
import sys

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
sys.path.insert(0, ROOT)

import bench  # noqa: E402
from nvfp4bench_b200.shard import shard_bounds  # noqa: E402


def test_configs_cover_the_baseline_workloads():
    for name in ("c1", "c2", "c3", "c3-16k", "c4"):
        assert name in bench.CONFIGS
    for m in (16, 64, 128):
        for kind in ("up", "down"):
            M, N, K, od, _ = bench.CONFIGS[f"decode-{kind}-{m}"]
            assert M == m and {N, K} == {14336, 4096} and od == "bf16"
    assert bench.CONFIGS["c4"][:3] == (4096, 14336, 8192)


def test_algorithmic_bytes():
    # C2: A 8.39 MB + SFA 1.05 + B 29.36 + SFB 3.67 + C (bf16) 117.44 = 159.9 MB
    assert abs(bench.algorithmic_bytes(4096, 14336, 4096, 2) - 159.9e6) < 0.1e6
    # sparse A: kept values K/4 + metadata K/16 + scales K/32 per row; B scales K/32
    M, N, K = 4096, 14336, 8192
    dense = bench.algorithmic_bytes(M, N, K, 2)
    sparse = bench.algorithmic_bytes(M, N, K, 2, sparse=True)
    assert sparse == M * K / 4 + M * K / 16 + M * K / 32 + N * K / 2 + N * K / 32 + M * N * 2
    assert sparse < dense


def test_strong_config_shards_evenly():
    M, N, K, _, _ = bench.CONFIGS["c3-16k"]
    assert "c3-16k" in bench.STRONG
    for g in (1, 2, 4, 8):
        widths = {n1 - n0 for n0, n1 in (shard_bounds(N, g, r) for r in range(g))}
        assert widths == {N // g}


def test_cpu_sample_counts_the_columns_it_ran():
    # The weight is capped at CPU_MAX_N columns; the FLOPs and the label must use that width.
    r = bench.cpu_reference_sample(64, bench.CPU_MAX_N + 4096, 256, target_s=0.05, threads=2)
    assert r["cols"] == bench.CPU_MAX_N
    assert r["flops"] == 2.0 * r["rows"] * r["cols"] * 256
    assert abs(r["tflops"] - r["flops"] / r["seconds"] / 1e12) < 1e-12
    assert f"x {bench.CPU_MAX_N} of {bench.CPU_MAX_N + 4096} cols" in r["sample"]
    assert r["rows"] <= 64


def test_reference_arm_line(capsys):
    rc = bench.main(["--impl", "reference", "--config", "c1", "--steps", "1", "--warmup", "0",
                     "--ref-step-s", "0.05"])
    assert rc == 0
    import json
    line = json.loads(capsys.readouterr().out.strip().splitlines()[-1])
    assert line["impl"] == "reference" and line["cpu_baseline"]["value"] == line["value"]
    assert line["e2e"]["h2d_bytes_per_step"] == 0
