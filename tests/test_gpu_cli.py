"""GPU: the C++ harness (bin/nvfp4bench, the counterpart of the reference's main.cu/bench.cu)
validates the b200 backend against its GPU FP32 oracle and reports the roofs."""
import json
import os
import subprocess

import pytest

from nvfp4bench_b200 import build

pytestmark = pytest.mark.gpu


def _run(args, tmp_path=None):
    if not os.path.exists(build.CLI):
        build.build()
    r = subprocess.run([build.CLI, *args], capture_output=True, text=True, timeout=300)
    return r


@pytest.mark.parametrize("args", [
    ["--m", "1024", "--n", "1024", "--k", "1024"],
    ["--m", "512", "--n", "768", "--k", "2048", "--out", "bf16", "--sf", "canonical"],
    ["--m", "300", "--n", "520", "--k", "288", "--dist", "uniform"],
    ["--m", "16", "--n", "4096", "--k", "14336", "--out", "bf16"],
    ["--m", "1024", "--n", "2048", "--k", "1024", "--cta-group", "2"],
    ["--m", "512", "--n", "640", "--k", "1024", "--mode", "sparse"],
    ["--m", "300", "--n", "384", "--k", "640", "--mode", "sparse", "--out", "bf16", "--sf", "canonical"],
])
def test_cli_validate(args, tmp_path):
    js = tmp_path / "r.json"
    r = _run([*args, "--validate", "--iters", "3", "--warmup", "1", "--json", str(js)])
    assert r.returncode == 0, r.stdout + r.stderr
    res = json.loads(js.read_text())["results"][0]
    assert res["ok"] and res["validated"] and res["pass"], r.stdout


def test_cli_reference_backends_not_built():
    r = _run(["--kernel", "all", "--m", "256", "--n", "256", "--k", "256", "--iters", "2"])
    assert r.returncode == 0
    assert "not run" in r.stdout and "b200" in r.stdout


def test_cli_roofs():
    r = _run(["--peak", "--bandwidth"])
    assert r.returncode == 0, r.stderr
    assert "TFLOPS" in r.stdout and "GB/s" in r.stdout


def test_cli_reports_nvml_clocks():
    """The device line carries the SM clocks read through NVML (reading only), as the
    reference's probe_device does (src/device_probe.cu:13-32)."""
    r = _run(["--kernel", "b200", "--m", "256", "--n", "256", "--k", "256", "--iters", "2"])
    assert r.returncode == 0, r.stdout + r.stderr
    line = [ln for ln in r.stdout.splitlines() if ln.startswith("SM clock (NVML)")]
    assert line, r.stdout
    if "unavailable" not in line[0]:
        mx = int(line[0].split("max ")[1].split(" MHz")[0])
        assert 1000 <= mx <= 3000, line[0]


def test_cli_csv_report(tmp_path):
    """--csv writes the reference's report columns (src/bench.cu:154-164) plus the roofline
    ones, one row per (kernel, shape, mode)."""
    import csv
    out = tmp_path / "r.csv"
    r = _run(["--kernel", "b200", "--mode", "both", "--m", "512", "--n", "640", "--k", "1024",
              "--validate", "--iters", "3", "--warmup", "1", "--csv", str(out)])
    assert r.returncode == 0, r.stdout + r.stderr
    rows = list(csv.DictReader(out.open()))
    assert [row["mode"] for row in rows] == ["dense", "2:4"], rows
    for row in rows:
        assert row["kernel"] == "b200" and (row["M"], row["N"], row["K"]) == ("512", "640", "1024")
        assert float(row["sust_tflops"]) > 0 and float(row["min_ms"]) > 0
        assert row["validated"] == "1" and row["pass"] == "1", row
        assert float(row["err_over_cinf"]) <= 1e-3  # FP32 output: the GEMM criterion
