"""Build the reference's own benchmark harness (src/main.cu + src/bench.cu and what they call)
against this engine: the recipe of INTEGRATION.md section 1, applied at build time.

    python nvfp4bench_b200/refharness/patch.py <reference project root>

The reference's sources are read from its tree and written, with the drop-in patch applied,
into _build/refharness/ (git-ignored; nothing of the reference enters this repository). Its
src/common.h and src/gemm.h are NOT copied: the harness compiles against this repository's
include/common.h and include/gemm.h, which keep the reference's types and fields and add
KernelKind::B200, launch_gemm_b200 and the defaulted operand extensions. The binary,
nvfp4bench_b200/bin/nvfp4bench_ref, links libnvfp4_b200.so and runs the reference's
run_bench (src/bench.cu:53-127) with `--kernel b200`.

The patch, each edit an exact text replacement that must match once:
  src/main.cu:93-97   `--kernel b200` selects KernelKind::B200 (also in the usage text).
  src/bench.cu:25-32  B is built N x K for the b200 backend (the layout of every BASELINE
                      config and of the reference's own CUTLASS/custom backends); the stub
                      keeps the K x N layout it reads.
  src/bench.cu:105-113 --validate also checks b200 against the reference's FP32 oracle
                      (src/reference.cu), given B transposed back to K x N.
"""
from __future__ import annotations

import os
import shutil
import subprocess
import sys

HERE = os.path.dirname(os.path.abspath(__file__))
PKG = os.path.dirname(HERE)
ROOT = os.path.dirname(PKG)
BUILD = os.path.join(ROOT, "_build", "refharness")
OUT = os.path.join(PKG, "bin", "nvfp4bench_ref")
LIB_DIR = os.path.join(PKG, "lib")

SOURCES = ["main.cu", "bench.cu", "nvfp4.cu", "reference.cu", "device_probe.cu", "peak.cu",
           "bandwidth.cu", "gemm_stub.cu"]
HEADERS = ["bench.h", "nvfp4.h", "reference.h", "device_probe.h", "peak.h"]

PATCHES = {
    "main.cu": [
        ('  if (want("custom"))  kernels.push_back(KernelKind::Custom);\n',
         '  if (want("custom"))  kernels.push_back(KernelKind::Custom);\n'
         '  if (want("b200"))    kernels.push_back(KernelKind::B200);\n'),
        ("--kernel  stub|cutlass|custom|all", "--kernel  stub|cutlass|custom|b200|all"),
    ],
    "bench.cu": [
        ("                              bool keep_host_dequant) {",
         "                              bool keep_host_dequant, bool b_nk = false) {"),
        ("  std::vector<float> Bh = make_random_matrix(p.k, p.n, cfg.seed ^ 0xABCDEF);",
         "  std::vector<float> Bh = b_nk ? make_random_matrix(p.n, p.k, cfg.seed ^ 0xABCDEF)\n"
         "                              : make_random_matrix(p.k, p.n, cfg.seed ^ 0xABCDEF);"),
        ("  Bt = quantize_to_nvfp4(Bh, p.k, p.n);",
         "  Bt = b_nk ? quantize_to_nvfp4(Bh, p.n, p.k) : quantize_to_nvfp4(Bh, p.k, p.n);"),
        ("upload_operands(prob, cfg, At, Bt, Adq, Bdq, cfg.validate);",
         "upload_operands(prob, cfg, At, Bt, Adq, Bdq, cfg.validate,\n"
         "                                     kind == KernelKind::B200);"),
        ("  if (cfg.validate && kind == KernelKind::Stub) {",
         "  if (cfg.validate && (kind == KernelKind::Stub || kind == KernelKind::B200)) {"),
        ("    std::vector<float> Cref = reference_gemm_fp32(Adq, Bdq, prob.m, prob.n, prob.k);",
         "    std::vector<float> Bkn = Bdq;\n"
         "    if (kind == KernelKind::B200)\n"
         "      for (int n_ = 0; n_ < prob.n; ++n_)\n"
         "        for (int k_ = 0; k_ < prob.k; ++k_)\n"
         "          Bkn[size_t(k_) * prob.n + n_] = Bdq[size_t(n_) * prob.k + k_];\n"
         "    std::vector<float> Cref = reference_gemm_fp32(Adq, Bkn, prob.m, prob.n, prob.k);"),
    ],
}


def nvcc() -> str:
    for cand in (os.environ.get("NVCC"), shutil.which("nvcc"), "/usr/local/cuda/bin/nvcc"):
        if cand and os.path.exists(cand):
            return cand
    raise FileNotFoundError("nvcc not found")


def stage(ref_src: str) -> None:
    """Copy the harness sources into BUILD with the patch applied."""
    os.makedirs(BUILD, exist_ok=True)
    for f in SOURCES + HEADERS:
        with open(os.path.join(ref_src, f)) as fh:
            text = fh.read()
        for old, new in PATCHES.get(f, []):
            if text.count(old) != 1:
                raise RuntimeError(f"patch text not found exactly once in {f}: {old[:60]!r}")
            text = text.replace(old, new)
        with open(os.path.join(BUILD, f), "w") as fh:
            fh.write(text)
    for f in ("common.h", "gemm.h"):  # the engine's versions of these must be the ones used
        p = os.path.join(BUILD, f)
        if os.path.exists(p):
            os.remove(p)


def build(ref_root: str) -> str:
    ref_src = os.path.join(ref_root, "src")
    stage(ref_src)
    lib = os.path.join(LIB_DIR, "libnvfp4_b200.so")
    if not os.path.exists(lib):
        raise FileNotFoundError(f"{lib} missing: build the engine first")
    os.makedirs(os.path.dirname(OUT), exist_ok=True)
    cuda = os.path.dirname(os.path.dirname(nvcc()))
    cmd = [nvcc(), "-gencode", "arch=compute_100a,code=sm_100a", "-O2", "-std=c++17",
           "-I", os.path.join(ROOT, "include"), "-I", BUILD,
           *[os.path.join(BUILD, f) for f in SOURCES],
           "-o", OUT, "-L", LIB_DIR, "-lnvfp4_b200",
           "-L", os.path.join(cuda, "lib64", "stubs"), "-lnvidia-ml",
           "-Xlinker", "-rpath=$ORIGIN/../lib"]
    r = subprocess.run(cmd, capture_output=True, text=True)
    if r.returncode != 0:
        raise RuntimeError("reference harness build failed:\n" + r.stdout + r.stderr)
    return OUT


def find_reference() -> str | None:
    """The reference project root: NVFP4BENCH_REF, else a checkout named `reference` beside
    this repository; None when neither has src/main.cu."""
    cands = [os.environ.get("NVFP4BENCH_REF"), os.path.join(os.path.dirname(ROOT), "reference")]
    for c in cands:
        if c and os.path.isfile(os.path.join(c, "src", "main.cu")):
            return c
    return None


if __name__ == "__main__":
    root = sys.argv[1] if len(sys.argv) > 1 else find_reference()
    if not root:
        sys.exit("reference tree not found: pass its root or set NVFP4BENCH_REF")
    print(build(root))
