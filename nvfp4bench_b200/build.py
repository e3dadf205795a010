"""Build the engine in-tree: nvfp4bench_b200/lib/libnvfp4_b200.so (C ABI, all CUDA kernels,
sm_100a only) and the C++ harness binary nvfp4bench_b200/bin/nvfp4bench.

    python -m nvfp4bench_b200.build [--verbose]

nvcc cross-compiles for sm_100a without a GPU. Objects go to _build/ (git-ignored).
"""
from __future__ import annotations

import argparse
import concurrent.futures as cf
import os
import shutil
import subprocess
import sys

PKG = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(PKG)
CSRC = os.path.join(PKG, "csrc")
HOST = os.path.join(CSRC, "host")
INCLUDE = os.path.join(ROOT, "include")
BUILD = os.path.join(ROOT, "_build")
LIB_DIR = os.path.join(PKG, "lib")
BIN_DIR = os.path.join(PKG, "bin")
LIB = os.path.join(LIB_DIR, "libnvfp4_b200.so")
CLI = os.path.join(BIN_DIR, "nvfp4bench")

ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]
NVCC_FLAGS = ["-O3", "-std=c++17", "-lineinfo", "-Xcompiler", "-fPIC", "-Xptxas", "-v",
              "--expt-relaxed-constexpr", "-I", INCLUDE, "-I", CSRC]
LIB_SOURCES = ["gemm_b200.cu", "gemm_noalloc.cu", "gemm_decode.cu", "codec.cu", "roofs.cu", "capi.cu",
               "ipc.cu"]


def nvcc() -> str:
    for cand in (os.environ.get("NVCC"), shutil.which("nvcc"), "/usr/local/cuda/bin/nvcc"):
        if cand and os.path.exists(cand):
            return cand
    raise FileNotFoundError("nvcc not found")


def _compile(src: str, obj: str, verbose: bool) -> str:
    cmd = [nvcc(), *ARCH, *NVCC_FLAGS, "-c", src, "-o", obj]
    r = subprocess.run(cmd, capture_output=True, text=True)
    if r.returncode != 0:
        raise RuntimeError(f"nvcc failed for {src}:\n{r.stdout}\n{r.stderr}")
    log = r.stdout + r.stderr
    if verbose:
        print(log)
    return log


def _stale(target: str, deps) -> bool:
    if not os.path.exists(target):
        return True
    t = os.path.getmtime(target)
    return any(os.path.getmtime(d) > t for d in deps)


def _headers():
    hs = []
    for d in (CSRC, INCLUDE, HOST):
        if os.path.isdir(d):
            hs += [os.path.join(d, f) for f in os.listdir(d) if f.endswith((".h", ".cuh"))]
    return hs


def build(verbose: bool = False, force: bool = False) -> str:
    os.makedirs(BUILD, exist_ok=True)
    os.makedirs(LIB_DIR, exist_ok=True)
    os.makedirs(BIN_DIR, exist_ok=True)
    headers = _headers()
    jobs = []
    objs = []
    for s in LIB_SOURCES:
        src = os.path.join(CSRC, s)
        obj = os.path.join(BUILD, s + ".o")
        objs.append(obj)
        if force or _stale(obj, [src, *headers]):
            jobs.append((src, obj))
    logs = {}
    with cf.ThreadPoolExecutor(max_workers=min(8, max(1, len(jobs)))) as ex:
        futs = {ex.submit(_compile, s, o, verbose): s for s, o in jobs}
        for f in cf.as_completed(futs):
            logs[futs[f]] = f.result()
    if force or _stale(LIB, objs):
        cmd = [nvcc(), *ARCH, "-shared", "-o", LIB, *objs, "-Xcompiler", "-fPIC",
               "-cudart", "static", "-lpthread", "-ldl", "-lrt"]
        r = subprocess.run(cmd, capture_output=True, text=True)
        if r.returncode != 0:
            raise RuntimeError(f"link failed:\n{r.stdout}\n{r.stderr}")
    # C++ harness (the reference's main.cu/bench.cu counterpart) over the C++ interface.
    host_srcs = sorted(os.path.join(HOST, f) for f in os.listdir(HOST) if f.endswith(".cpp")) \
        if os.path.isdir(HOST) else []
    if host_srcs and (force or _stale(CLI, [*host_srcs, LIB, *headers])):
        cmd = [nvcc(), *ARCH, "-O2", "-std=c++17", "-I", INCLUDE, "-I", CSRC, *host_srcs,
               "-o", CLI, "-L", LIB_DIR, "-lnvfp4_b200", "-Xlinker", "-rpath,$ORIGIN/../lib",
               "-cudart", "static", "-lpthread", "-ldl", "-lrt"]
        r = subprocess.run(cmd, capture_output=True, text=True)
        if r.returncode != 0:
            raise RuntimeError(f"harness build failed:\n{r.stdout}\n{r.stderr}")
    # The reference's own harness linked against this library,
    # where the reference tree is at hand; the binary then travels with the repository.
    import importlib.util
    spec = importlib.util.spec_from_file_location(
        "nvfp4_refharness", os.path.join(PKG, "refharness", "patch.py"))
    rh = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(rh)
    ref = rh.find_reference()
    if ref and (force or _stale(rh.OUT, [LIB, os.path.join(PKG, "refharness", "patch.py"),
                                         *headers])):
        rh.build(ref)
    if logs:
        with open(os.path.join(BUILD, "ptxas.log"), "w") as f:
            for k in sorted(logs):
                f.write(f"== {k}\n{logs[k]}\n")
    return LIB


def main(argv=None) -> int:
    ap = argparse.ArgumentParser()
    ap.add_argument("--verbose", action="store_true")
    ap.add_argument("--force", action="store_true")
    a = ap.parse_args(argv)
    print(build(verbose=a.verbose, force=a.force))
    return 0


if __name__ == "__main__":
    sys.exit(main())
