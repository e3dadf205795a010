#!/usr/bin/env python
"""Benchmark of the NVFP4 GEMM hot path (BASELINE.json metric: NVFP4 GEMM TFLOPS at
4096x14336x4096 and % of the measured tcgen05 FP4 peak).

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl b200|reference]
                    [--config c2|c1|c3|c3-16k|c4|decode-{up,down}-{16,64,128}]
                    [--gather] [--quantize-a] [--b-static] [--kernel-only]
                    [--no-cpu-baseline] [--no-extras] [--extra-steps S]

One step = one D = A*B^T launch of the workload (config 2 of BASELINE.json by default:
M=4096 tokens, N=14336, K=4096, N(0,1) operands quantised on the GPU to E2M1/UE4M3, BF16 out).
c4 is the pair-wise 2:4 sparse configuration (the format the tcgen05 .sp MMA executes);
decode-* are the M <= 128 weight-streaming shapes. Under torchrun every rank computes its own
N-slice of a problem N*world wide (weak scaling, no data-path collective), except c3-16k,
whose N = 65536 is split over the ranks (strong scaling). At N > 1 the line also times the
optional all-gather of the C shards (`gather`; --no-gather skips it), both as NCCL all-gather +
row-major copy after the GEMM and fused into the GEMM's epilogue (tiles stored straight into
every rank's row-major output over NVLink), each against the measured NVLink rate.
Rank 0 prints one JSON line. At N=1 the line also carries `extra`: every other BASELINE
configuration that fits one GPU (C1, C2 with canonical scales, C3 8192^3, C4, the six
decode shapes), each timed under the same rules with its own roofline fraction; `gpu_launches`
counts the headline's timed region only.

`value` is device-timed with operands resident in HBM: for M > 128 the L2 is flushed (256 MiB
write) before every step and CUDA events bracket each launch; decode shapes rotate the weight
over copies larger than 3x L2 and time the K back-to-back steps with one event pair (the next
launch's prologue overlaps through programmatic dependent launch); max over ranks. Decode
shapes are also timed as replays of one captured CUDA graph of >= 100 launches (`graph`).
--quantize-a adds the GPU quantisation of fp32 A to every (decode) step. `e2e` is the same
metric through the C ABI with pinned host buffers: each step copies the quantised operands
host->device, launches, and copies C device->host, all inside the timed region (consecutive
steps pipelined over three streams, as a serving loop would run them).
`--impl reference` times the reference's own algorithm for this path on the host cores (the
CPU restatement of src/reference.cu in oracle/, over dequantised operands) on a bounded
sample of output rows; it never touches the GPU.
"""
from __future__ import annotations

import argparse
import json
import os
import statistics
import subprocess
import sys
import threading
import time

import numpy as np

ROOT = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, ROOT)

CONFIGS = {
    # name: (M, N, K, out dtype, description)
    "c1": (1024, 1024, 1024, "f32", "NVFP4 GEMM 1024^3, FP32 out (BASELINE config 1)"),
    "c2": (4096, 14336, 4096, "bf16", "LLM FFN up-proj 4096x14336x4096, BF16 out (BASELINE config 2)"),
    # BASELINE config 3's large case: N = 65536 split over the ranks (strong scaling).
    "c3-16k": (16384, 65536, 16384, "bf16", "16384x65536x16384, BF16 out, N split over the GPUs (BASELINE config 3)"),
    # BASELINE config 4 as the tcgen05 .sp kind::mxf4nvf4 MMA executes it on B200: 2 of the 4
    # element pairs of every 8 K elements of A kept (seeded), UE4M3 scales per 32 K.
    "c4": (4096, 14336, 8192, "bf16", "pair-wise 2:4 sparse NVFP4 4096x14336x8192, BF16 out (BASELINE config 4)"),
    "c3": (8192, 8192, 8192, "bf16", "square 8192^3, BF16 out (BASELINE config 3, 1 GPU)"),
    "decode-up-16": (16, 14336, 4096, "bf16", "decode M=16 up-proj"),
    "decode-up-64": (64, 14336, 4096, "bf16", "decode M=64 up-proj"),
    "decode-up-128": (128, 14336, 4096, "bf16", "decode M=128 up-proj"),
    "decode-down-16": (16, 4096, 14336, "bf16", "decode M=16 down-proj"),
    "decode-down-64": (64, 4096, 14336, "bf16", "decode M=64 down-proj"),
    "decode-down-128": (128, 4096, 14336, "bf16", "decode M=128 down-proj"),
}
SEED_A, SEED_B = 1234, 1234 ^ 0xABCDEF
SEED_SPARSE = 0x24  # pair pattern of the sparse config


# Configs whose N is the total over all ranks (strong scaling); the others give every rank its
# own N-wide slice of a world*N-wide weight (weak scaling).
STRONG = {"c3-16k"}
# NVLink peer copy measured on this pool, GB/s per direction per GPU (nominal 900).
LINK_GBS = 770.0
# The CPU baseline times a column sample of at most this many weight rows (its rate is per FLOP).
CPU_MAX_N = 8192


def algorithmic_bytes(M, N, K, out_bytes, sparse=False):
    """Operand values + scales read once, C written once (SURVEY roofline convention). Sparse:
    A's kept values K/4 B + metadata K/16 B + scales K/32 B per row, B's scales K/32 B."""
    if sparse:
        return M * K / 4 + M * K / 16 + M * K / 32 + N * K / 2 + N * K / 32 + M * N * out_bytes
    return M * K / 2 + M * K / 16 + N * K / 2 + N * K / 16 + M * N * out_bytes


# ------------------------------------------------------------------------------- clocks
class ClockSampler:
    """nvidia-smi samples during the timed region (clocks, power, throttle reasons)."""

    FIELDS = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
              "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
              "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, gpu_index: int):
        self.gpu = gpu_index
        self.proc = None
        self.lines = []
        self.thread = None

    def start(self):
        try:
            self.proc = subprocess.Popen(
                ["nvidia-smi", f"--id={self.gpu}", f"--query-gpu={self.FIELDS}",
                 "--format=csv,noheader,nounits", "-lms", "100"],
                stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
        except (FileNotFoundError, OSError):
            self.proc = None
            return
        self.thread = threading.Thread(target=self._read, daemon=True)
        self.thread.start()

    def _read(self):
        for line in self.proc.stdout:
            self.lines.append(line.strip())

    def stop(self):
        if self.proc is None:
            return None
        self.proc.terminate()
        try:
            self.proc.wait(timeout=5)
        except subprocess.TimeoutExpired:
            self.proc.kill()
        if self.thread:
            self.thread.join(timeout=2)
        sm, smax, reasons = [], [], set()
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        for ln in self.lines:
            parts = [p.strip() for p in ln.split(",")]
            if len(parts) < 9:
                continue
            try:
                sm.append(float(parts[1]))
                smax.append(float(parts[2]))
            except ValueError:
                continue
            for n, v in zip(names, parts[5:9]):
                if v.lower().startswith("active"):
                    reasons.add(n)
        if not sm:
            return None
        return {"sm_mhz": statistics.median(sm), "sm_max_mhz": max(smax) if smax else None,
                "reasons": sorted(reasons), "samples": len(sm)}


# ------------------------------------------------------------------------------- reference arm
def cpu_reference_sample(M, N, K, target_s, threads=0):
    """Time the oracle (CPU restatement of src/reference.cu:9-17) on a seeded sample of the
    workload: a column slice of at most CPU_MAX_N weight rows and as many output rows as fit in
    about `target_s` seconds. Returns a dict with the rate and exactly what ran (the FLOPs are
    counted over the columns that ran, not the workload's full N)."""
    import oracle
    rng = np.random.default_rng(SEED_A)
    n_cols = min(N, CPU_MAX_N)
    a_rows = min(M, 256)
    # N(0,1) operands of the workload's distribution (numpy-seeded), quantised and dequantised
    # by the oracle: the values the reference's oracle would consume.
    a = rng.standard_normal((a_rows, K), dtype=np.float32)
    b = np.random.default_rng(SEED_B).standard_normal((n_cols, K), dtype=np.float32)
    pa, sa = oracle.quantize(a)
    pb, sb = oracle.quantize(b)
    adq = oracle.dequantize(pa, sa, K)
    bdq = oracle.dequantize(pb, sb, K)
    nthreads = threads if threads > 0 else oracle.default_threads()
    # Calibrate: rows per second with all threads.
    probe = max(nthreads, 8)
    rows = rng.integers(0, a_rows, probe).astype(np.int32)
    t0 = time.perf_counter()
    oracle.gemm_nt_rows(adq, bdq, rows, threads=nthreads)
    dt = time.perf_counter() - t0
    n_rows = max(nthreads, int(probe * target_s / max(dt, 1e-6)))
    n_rows = min(n_rows, M)
    rows = rng.integers(0, a_rows, n_rows).astype(np.int32)
    t0 = time.perf_counter()
    oracle.gemm_nt_rows(adq, bdq, rows, threads=nthreads)
    dt = time.perf_counter() - t0
    flops = 2.0 * n_rows * n_cols * K
    return {"tflops": flops / dt / 1e12, "rows": n_rows, "cols": n_cols, "flops": flops,
            "seconds": dt, "threads": nthreads, "distinct_rows": a_rows,
            "sample": (f"{n_rows} output rows (drawn from {a_rows} distinct seeded N(0,1) A rows) "
                       f"x {n_cols} of {N} cols, K={K}; naive FP32 k-ascending oracle "
                       f"(src/reference.cu restated) on dequantised NVFP4 operands, "
                       f"{nthreads} host threads")}


def run_reference(args, rank, world):
    cfg = CONFIGS[args.config]
    M, N, K, od, desc = cfg
    if rank != 0:
        return 0
    per_step = []
    for i in range(args.warmup + args.steps):
        r = cpu_reference_sample(M, N, K, target_s=args.ref_step_s)
        if i >= args.warmup:
            per_step.append(r)
    tot_flops = sum(r["flops"] for r in per_step)
    tot_t = sum(r["seconds"] for r in per_step)
    val = tot_flops / tot_t / 1e12
    last = per_step[-1]
    line = {
        "impl": "reference", "metric": "nvfp4_gemm_tflops", "value": val, "unit": "TFLOP/s",
        "n_gpus": world, "steps": args.steps, "warmup": args.warmup,
        "ms_per_step": 1e3 * tot_t / len(per_step), "higher_is_better": True,
        "scaling": "weak", "vs_baseline": None, "dtype": "f32", "data": "synthetic",
        "config": {"workload": desc, "M": M, "N": N, "K": K},
        "cpu_baseline": {"value": val, "unit": "TFLOP/s", "cores": last["threads"], "kind": "port",
                         "sample": "per step: " + last["sample"]},
        "e2e": {"value": val, "unit": "TFLOP/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }
    print(json.dumps(line), flush=True)
    return 0


# ------------------------------------------------------------------------------- extra configs
# Every other BASELINE configuration that fits one GPU, timed in the default (N=1) run beside
# the headline: C1 (1024^3, FP32 out), C2 with canonical [rows][K/16] scales (the layout the
# reference harness hands over, so each call also reorders them), C3 8192^3, C4 and the six
# decode shapes.
EXTRA_CONFIGS = ("c1", "c2-canonical", "c3", "c4", "decode-up-16", "decode-up-64", "decode-up-128",
                 "decode-down-16", "decode-down-64", "decode-down-128")


def graph_ms_per_launch(api, rot, stream, dev, replays=3):
    """Per-launch time of a captured CUDA graph of >= 100 launches over the argument blocks
    `rot` (the rotated weight copies; programmatic dependent launch edges between them),
    replayed `replays` times between one event pair on `stream`. Returns (ms, launches)."""
    import torch
    n_launch = -(-100 // len(rot)) * len(rot)
    g = torch.cuda.CUDAGraph()
    cap = torch.cuda.Stream(dev)
    cap.wait_stream(stream)
    with torch.cuda.stream(cap):
        with torch.cuda.graph(g, stream=cap):
            for i in range(n_launch):
                api.launch(rot[i % len(rot)])
    stream.wait_stream(cap)
    g.replay()
    torch.cuda.synchronize()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    torch.cuda._sleep(100_000)
    e0.record(stream)
    for _ in range(replays):
        g.replay()
    e1.record(stream)
    torch.cuda.synchronize()
    ms = e0.elapsed_time(e1) / (replays * n_launch)
    del g
    return ms, n_launch


def time_extra(api, name, dev, steps, ladder, hbm_gbs):
    """Operands for workload `name` made and quantised on the GPU, then `steps` timed steps
    under the headline's rules: M > 128 flushes L2 (256 MiB write) before each step and times
    it with its own event pair; decode shapes rotate the weight over copies holding >= 3x L2
    and time the steps back to back. Returns a compact result dict."""
    import torch
    canonical = name.endswith("-canonical")
    cfg = name[: -len("-canonical")] if canonical else name
    M, N, K, od, desc = CONFIGS[cfg]
    out_dtype = torch.bfloat16 if od == "bf16" else torch.float32
    out_bytes = 2 if od == "bf16" else 4
    sparse = cfg == "c4"
    x = api.fill_normal(M, K, SEED_A)
    a_meta = None
    if sparse:
        a_meta = api.sparse_meta(M, K, SEED_SPARSE)
        api.sparse_prune(x, a_meta)
        A = api.quantize_block(x, 32, canonical=False, tcgen05=True)
        A.packed = api.sparse_compress(A.packed, a_meta, K)
    else:
        A = api.quantize(x, canonical=canonical, tcgen05=not canonical)
    del x
    x = api.fill_normal(N, K, SEED_B)
    B = (api.quantize_block(x, 32, canonical=False, tcgen05=True) if sparse else
         api.quantize(x, canonical=canonical, tcgen05=not canonical))
    del x
    C = torch.empty((M, N), dtype=out_dtype, device=dev)
    mode = api.MODE_SPARSE24 if sparse else api.MODE_DENSE
    sfl = api.SF_CANONICAL if canonical else api.SF_TCGEN05

    def scales(t):
        return t.scales if canonical else t.scales_tc

    decode = M <= 128
    rot = [api.gemm_args(A.packed, scales(A), B.packed, scales(B), M, N, K, C, sf_layout=sfl,
                         mode=mode, a_meta=a_meta)]
    keep = []
    if decode:
        wbytes = B.packed.numel() + scales(B).numel()
        for _ in range(max(2, -(-3 * 126_000_000 // wbytes)) - 1):
            bp, bs = B.packed.clone(), scales(B).clone()
            keep.append((bp, bs))
            rot.append(api.gemm_args(A.packed, scales(A), bp, bs, M, N, K, C, sf_layout=sfl))
    flush = None if decode else torch.empty(256 << 20, dtype=torch.uint8, device=dev)
    stream = torch.cuda.current_stream()
    i = [0]

    def step():
        api.launch(rot[i[0] % len(rot)])
        i[0] += 1

    for _ in range(max(3, 2 * len(rot))):
        if flush is not None:
            flush.zero_()
        step()
    torch.cuda.synchronize()
    torch.cuda._sleep(steps * (100_000 if decode else 300_000))
    if decode:
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record(stream)
        for _ in range(steps):
            step()
        e1.record(stream)
        torch.cuda.synchronize()
        ms = e0.elapsed_time(e1) / steps
    else:
        ev = [(torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True))
              for _ in range(steps)]
        for s_, e_ in ev:
            flush.zero_()
            s_.record(stream)
            step()
            e_.record(stream)
        torch.cuda.synchronize()
        ms = sum(s_.elapsed_time(e_) for s_, e_ in ev) / steps
    g_ms = graph_ms_per_launch(api, rot, stream, dev)[0] if decode else None
    if api.device_error():
        raise RuntimeError(f"{name}: device error word set")
    flops = 2.0 * M * N * K
    abytes = algorithmic_bytes(M, N, K, out_bytes, sparse)
    r = {"workload": desc + (" (canonical scales, reordered every call)" if canonical else ""),
         "M": M, "N": N, "K": K, "ms_per_step": ms, "tflops": flops / (ms * 1e-3) / 1e12,
         "gbs": abytes / (ms * 1e-3) / 1e9, "algorithmic_bytes": abytes,
         "gpu_launches_per_step": 2 if canonical else 1,
         "l2": ("weight rotated over %d copies (> 3x L2)" % len(rot)) if decode else
               "flushed before every step"}
    if decode:
        r["roofline"] = {"bound": "hbm", "peak": hbm_gbs, "unit": "GB/s",
                         "frac": r["gbs"] / hbm_gbs, "peak_source": "MEASURED_PEAKS.json hbm_gbs"}
        # The same launches replayed from one CUDA graph (>= 100 per replay).
        r["graph"] = {"ms_per_step": g_ms, "gbs": abytes / (g_ms * 1e-3) / 1e9,
                      "frac": abytes / (g_ms * 1e-3) / 1e9 / hbm_gbs}
    else:
        key = "sparse_random_burst" if sparse else "random_burst"
        peak = (ladder.get(key) or {}).get("tflops")
        r["roofline"] = {"bound": "tensor", "peak": peak, "unit": "TFLOP/s",
                         "frac": r["tflops"] / peak if peak else None,
                         "peak_source": "tcgen05 FP4 ladder rung '%s' of this run" % key}
    del keep, rot, A, B, C, flush
    torch.cuda.empty_cache()
    return r


def run_extras(api, dev, steps, ladder, hbm_gbs, gpu_index):
    """Time EXTRA_CONFIGS one after another; one clock record covers them all."""
    clocks = ClockSampler(gpu_index)
    clocks.start()
    time.sleep(0.3)
    res = {}
    for name in EXTRA_CONFIGS:
        res[name] = time_extra(api, name, dev, steps, ladder, hbm_gbs)
    res["clocks"] = clocks.stop()
    return res


# ------------------------------------------------------------------------------- b200 arm
def run_b200(args, rank, world, local_rank):
    import torch
    import torch.distributed as dist
    from nvfp4bench_b200 import api
    from nvfp4bench_b200.shard import max_over_ranks, shard_bounds

    torch.cuda.set_device(local_rank)
    dev = torch.device("cuda", local_rank)
    M, N, K, od, desc = CONFIGS[args.config]
    out_dtype = torch.bfloat16 if od == "bf16" else torch.float32
    out_bytes = 2 if od == "bf16" else 4
    stream = torch.cuda.current_stream()

    # Operands: A replicated (same seed on every rank), B = this rank's N-slice [n0, n1) of a
    # world*N-wide weight (weak scaling) or of the config's N-wide weight (strong scaling),
    # drawn with the weight seed offset by the rank.
    strong = args.config in STRONG
    n_total = N if strong else world * N
    n0, n1 = shard_bounds(n_total, world, rank)
    N = n1 - n0
    if max_over_ranks([N], device=dev)[0] != N:
        raise RuntimeError("strong scaling needs equal shards: N must divide over the ranks in 128-row blocks")
    sparse = args.config == "c4"
    x = api.fill_normal(M, K, SEED_A)
    a_meta = None
    if sparse:
        # Seeded pair pattern, pruned, quantised with 32-element scales, compressed.
        a_meta = api.sparse_meta(M, K, SEED_SPARSE)
        api.sparse_prune(x, a_meta)
        A = api.quantize_block(x, 32, canonical=False, tcgen05=True)
        A.packed = api.sparse_compress(A.packed, a_meta, K)
    else:
        A = api.quantize(x, canonical=False, tcgen05=True)
    del x
    x = api.fill_normal(N, K, SEED_B + rank)
    B = api.quantize_block(x, 32, canonical=False, tcgen05=True) if sparse else \
        api.quantize(x, canonical=False, tcgen05=True)
    del x
    C = torch.empty((M, N), dtype=out_dtype, device=dev)
    mode = api.MODE_SPARSE24 if sparse else api.MODE_DENSE
    # --quantize-a: the weights are never written by the quantisation that precedes each
    # GEMM, so the decode kernel may start streaming them before it completes (b_static).
    gargs = api.gemm_args(A.packed, A.scales_tc, B.packed, B.scales_tc, M, N, K, C,
                          sf_layout=api.SF_TCGEN05, tile_n=args.tile_n,
                          cta_group=args.cta_group, mode=mode, a_meta=a_meta,
                          b_static=args.quantize_a or args.b_static)
    flush = torch.empty(256 << 20, dtype=torch.uint8, device=dev)
    torch.cuda.synchronize()

    # Measured compute roofs for this run (tcgen05 FP4 ladder, M128 N256 K64 on every SM):
    # random E2M1 operands timed alone (the roof for this GEMM, which is timed alone), zero
    # operands (the issue-rate ceiling at full clock) and random operands back to back for
    # about a second (under the power cap); each with the SM clock it ran at.
    ladder = {}
    if not args.kernel_only:
        sms = torch.cuda.get_device_properties(dev).multi_processor_count
        # Burst rungs first: the sustained rung leaves the clock at its power-capped level.
        rungs = [("random_burst", 0x5EED, False, 5, False), ("zero_burst", 0, False, 5, False)]
        if sparse or (world == 1 and not args.no_extras):
            rungs.append(("sparse_random_burst", 0x5EED, False, 5, True))
        rungs.append(("random_sustained", 0x5EED, True, 2000, False))
        for key, seed, sustained, reps, sp in rungs:
            tf, mhz = api.peak_ex(256, 1, sms, 4096, reps, seed=seed, sustained=sustained, sparse=sp)
            ladder[key] = {"tflops": round(tf, 1), "sm_mhz": round(mhz)}
    peak_key = "sparse_random_burst" if sparse else "random_burst"
    peak_tf = ladder[peak_key]["tflops"] if ladder else None

    # Decode shapes (M <= 128) stream the weight once per step, and a flush that writes 256 MiB
    # leaves L2 full of dirty lines whose write-back competes with that stream. They use inputs
    # larger than L2 instead: the weight is rotated over R copies holding at least 3x L2, so
    # each step reads a weight that the steps since its last use have evicted.
    decode = M <= 128
    rot = [gargs]
    if decode:
        wbytes = B.packed.numel() + B.scales_tc.numel()
        copies = max(2, -(-3 * 126_000_000 // wbytes))
        keep = []
        for _ in range(copies - 1):
            bp, bs = B.packed.clone(), B.scales_tc.clone()
            keep.append((bp, bs))
            rot.append(api.gemm_args(A.packed, A.scales_tc, bp, bs, M, N, K, C,
                                     sf_layout=api.SF_TCGEN05, tile_n=args.tile_n,
                                     cta_group=args.cta_group,
                                     b_static=args.quantize_a or args.b_static))
    step_no = [0]
    # --quantize-a: every step quantises the fp32 activations A into the tcgen05-layout operand
    # the GEMM reads (the per-call cost of a real decode layer) and runs the GEMM, through
    # nvfp4_b200_gemm_quantize_a: one fused launch for decode shapes, the quantiser and the GEMM
    # back to back otherwise.
    xa = None
    if args.quantize_a:
        if sparse:
            raise SystemExit("--quantize-a applies to dense configs")
        xa = api.fill_normal(M, K, SEED_A)
    fused_qa = args.quantize_a and decode and K % 64 == 0

    def step():
        if xa is not None:
            api.launch_quantize_a(rot[step_no[0] % len(rot)], xa)
        else:
            api.launch(rot[step_no[0] % len(rot)])
        step_no[0] += 1

    def before_step():
        if not decode:
            flush.zero_()

    for _ in range(max(3, args.warmup, 2 * len(rot) if decode else 0)):
        before_step()
        step()
    torch.cuda.synchronize()
    if world > 1:
        dist.barrier()

    starts = [torch.cuda.Event(enable_timing=True) for _ in range(args.steps)]
    ends = [torch.cuda.Event(enable_timing=True) for _ in range(args.steps)]
    clocks = ClockSampler(local_rank) if rank == 0 else None
    if clocks:
        clocks.start()
        time.sleep(0.3)
    torch.cuda.synchronize()
    if world > 1:
        dist.barrier()
    # A GPU spin in front lets the host enqueue every step (flush, events, launch) before the
    # first one runs, so the events time the device and never a host launch gap: a decode step
    # is shorter than the host's launch path, and the flush in front of a large step can be too.
    torch.cuda._sleep(args.steps * (100_000 if decode else 300_000))
    if decode:
        # One event pair around the K back-to-back steps: an event between two launches
        # would stand between them and stop the next one's set-up from overlapping.
        starts[0].record(stream)
        for i in range(args.steps):
            step()
        ends[0].record(stream)
    else:
        for i in range(args.steps):
            before_step()
            starts[i].record(stream)
            step()
            ends[i].record(stream)
    torch.cuda.synchronize()
    if world > 1:
        dist.barrier()
    clk = clocks.stop() if clocks else None
    if decode:
        times = [starts[0].elapsed_time(ends[0]) / args.steps] * args.steps
    else:
        times = [s.elapsed_time(e) for s, e in zip(starts, ends)]
    mean_ms = sum(times) / len(times)
    min_ms, med_ms = min(times), statistics.median(times)
    mean_ms, min_ms, med_ms = max_over_ranks([mean_ms, min_ms, med_ms], device=dev)
    derr = api.device_error()
    if derr:
        raise RuntimeError(f"device error word {derr:#x}")

    # Decode shapes again from one captured CUDA graph: >= 100 launches over the rotated weight
    # copies (programmatic dependent launch edges between them), replayed three times between
    # one event pair - the form a serving loop would use. Reported beside the stream timing.
    graph = None
    if decode and xa is None:
        if world > 1:
            dist.barrier()
        g_ms, n_launch = graph_ms_per_launch(api, rot, stream, dev)
        g_ms = max_over_ranks([g_ms], device=dev)[0]
        derr = api.device_error()
        if derr:
            raise RuntimeError(f"device error word {derr:#x} (graph replay)")
        graph = {"ms_per_step": g_ms, "launches_per_replay": n_launch, "replays": 3,
                 "value": world * 2.0 * M * N * K / (g_ms * 1e-3) / 1e12}

    flops = 2.0 * M * N * K
    value = world * flops / (mean_ms * 1e-3) / 1e12
    achieved = flops / (mean_ms * 1e-3) / 1e12
    if args.kernel_only:
        if rank == 0:
            line = {"metric": "nvfp4_gemm_tflops", "value": value, "unit": "TFLOP/s",
                    "ms_per_step": mean_ms, "kernel_only": True, "config": {"workload": desc}}
            if graph:
                line["graph"] = graph
            print(json.dumps(line), flush=True)
        return 0

    # Reference-style timing (src/bench.cu:90-105): per-launch events, no flush, burst=min,
    # sustained=median of 50.
    ev = [(torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True))
          for _ in range(50)]
    if decode:
        torch.cuda._sleep(len(ev) * 100_000)
    for s_, e_ in ev:
        s_.record(stream)
        step()
        e_.record(stream)
    torch.cuda.synchronize()
    rt = sorted(s_.elapsed_time(e_) for s_, e_ in ev)
    burst_tf, sust_tf = flops / (rt[0] * 1e-3) / 1e12, flops / (rt[len(rt) // 2] * 1e-3) / 1e12

    # e2e through the C ABI with pinned host buffers: every step copies its quantised operands
    # host->device, launches, and copies C device->host. Consecutive steps are pipelined the
    # way a serving loop would run them: host->device copies on one stream, the GEMM on the
    # launch stream, device->host copies on a third, device buffers doubled, so step i+1's
    # inputs and step i-1's result cross PCIe (in opposite directions) while step i computes.
    hA, hAs = A.packed.cpu().pin_memory(), A.scales_tc.cpu().pin_memory()
    hB, hBs = B.packed.cpu().pin_memory(), B.scales_tc.cpu().pin_memory()
    hM = a_meta.cpu().pin_memory() if sparse else None
    hCs = [torch.empty((M, N), dtype=out_dtype).pin_memory() for _ in range(2)]
    dbuf = []
    for _ in range(2):
        d = {"A": torch.empty_like(A.packed), "As": torch.empty_like(A.scales_tc),
             "B": torch.empty_like(B.packed), "Bs": torch.empty_like(B.scales_tc),
             "M": torch.empty_like(a_meta) if sparse else None, "C": torch.empty_like(C)}
        d["args"] = api.gemm_args(d["A"], d["As"], d["B"], d["Bs"], M, N, K, d["C"],
                                  sf_layout=api.SF_TCGEN05, tile_n=args.tile_n,
                                  cta_group=args.cta_group, mode=mode, a_meta=d["M"])
        dbuf.append(d)
    h2d = hA.numel() + hAs.numel() + hB.numel() + hBs.numel() + (hM.numel() if sparse else 0)
    d2h = M * N * out_bytes
    s_in, s_out = torch.cuda.Stream(dev), torch.cuda.Stream(dev)
    ev_in = [torch.cuda.Event() for _ in range(2)]
    ev_gemm = [torch.cuda.Event() for _ in range(2)]
    ev_out = [torch.cuda.Event() for _ in range(2)]
    e2e_i = [0]

    def e2e_step():
        k = e2e_i[0] % 2
        d, hC = dbuf[k], hCs[k]
        with torch.cuda.stream(s_in):
            s_in.wait_event(ev_gemm[k])        # step i-2's GEMM has read these inputs
            d["A"].copy_(hA, non_blocking=True)
            d["As"].copy_(hAs, non_blocking=True)
            d["B"].copy_(hB, non_blocking=True)
            d["Bs"].copy_(hBs, non_blocking=True)
            if sparse:
                d["M"].copy_(hM, non_blocking=True)
            ev_in[k].record(s_in)
        stream.wait_event(ev_in[k])
        stream.wait_event(ev_out[k])           # step i-2's result has left this buffer
        api.launch(d["args"], stream)
        ev_gemm[k].record(stream)
        with torch.cuda.stream(s_out):
            s_out.wait_event(ev_gemm[k])
            hC.copy_(d["C"], non_blocking=True)
            ev_out[k].record(s_out)
        e2e_i[0] += 1

    for _ in range(2):
        e2e_step()
    torch.cuda.synchronize()
    if world > 1:
        dist.barrier()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record(stream)
    s_in.wait_event(e0)
    for _ in range(args.steps):
        e2e_step()
    for k in range(2):
        stream.wait_event(ev_out[k])
    e1.record(stream)
    torch.cuda.synchronize()
    e2e_ms = max_over_ranks([e0.elapsed_time(e1) / args.steps], device=dev)[0]
    hC = hCs[(e2e_i[0] - 1) % 2]
    if not torch.equal(hC.to(dev), C):
        raise RuntimeError("e2e output differs from the device-resident output")

    gather = None
    if world > 1 and not args.no_gather:
        # The optional exchange: one NCCL all-gather of the C column shards over NVLink, then
        # the optional copy into a row-major [M][N_total] matrix, each timed on its own.
        from nvfp4bench_b200.shard import gather_shards, shards_to_row_major
        shards = gather_shards(C, n_total)
        full = shards_to_row_major(shards, n_total)
        torch.cuda.synchronize()
        ev3 = [torch.cuda.Event(enable_timing=True) for _ in range(3)]
        dist.barrier()
        ev3[0].record(stream)
        for _ in range(args.steps):
            gather_shards(C, n_total, out=shards)
        ev3[1].record(stream)
        for _ in range(args.steps):
            shards_to_row_major(shards, n_total, out=full)
        ev3[2].record(stream)
        torch.cuda.synchronize()
        g_ms, r_ms = max_over_ranks([ev3[0].elapsed_time(ev3[1]) / args.steps,
                                     ev3[1].elapsed_time(ev3[2]) / args.steps], device=dev)
        moved = M * N * out_bytes * (world - 1)   # bytes each rank receives
        gather = {"ms_per_all_gather": g_ms, "bytes_received_per_gpu": moved,
                  "gbs_per_gpu": moved / (g_ms * 1e-3) / 1e9,
                  "ms_row_major_copy": r_ms, "full_shape": [int(full.shape[0]), int(full.shape[1])]}

        # The fused form: each rank's epilogue stores its tiles into every rank's row-major
        # [M][N_total] buffer over NVLink (CUDA IPC mappings) as they complete; a one-word NCCL
        # all-reduce per step orders all ranks' GEMMs before the result is read. Timed per
        # step (GEMM with its gather + that all-reduce) like the GEMM alone, L2 flushed.
        from nvfp4bench_b200.shard import GatheredOutput
        go = GatheredOutput(M, n_total, out_dtype, dev)
        if go.n1 - go.n0 != N:
            raise RuntimeError("shard width differs from the per-rank N")
        fargs = api.gemm_args(A.packed, A.scales_tc, B.packed, B.scales_tc, M, N, K, go.local,
                              sf_layout=api.SF_TCGEN05, tile_n=args.tile_n,
                              cta_group=args.cta_group, mode=mode, a_meta=a_meta,
                              peers=go.peers)
        for _ in range(max(3, args.warmup)):
            flush.zero_()
            api.launch(fargs)
            go.wait_all()
        torch.cuda.synchronize()
        identical = bool(torch.equal(go.full, full))
        fs = [(torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True))
              for _ in range(args.steps)]
        dist.barrier()
        for s_, e_ in fs:
            flush.zero_()
            s_.record(stream)
            api.launch(fargs)
            go.wait_all()
            e_.record(stream)
        torch.cuda.synchronize()
        f_ms = max_over_ranks([sum(s_.elapsed_time(e_) for s_, e_ in fs) / len(fs)], device=dev)[0]
        go.wait_all()
        torch.cuda.synchronize()
        dist.barrier()
        go.close()
        gather["link_peak_gbs"] = LINK_GBS
        gather["nccl_link_frac"] = moved / (g_ms * 1e-3) / 1e9 / LINK_GBS
        gather["fused"] = {
            "ms_per_step": f_ms,
            # Bytes each rank receives over NVLink per step against the link's measured rate:
            # the fused step cannot beat max(GEMM time, bytes / link rate).
            "link_frac": moved / (f_ms * 1e-3) / 1e9 / LINK_GBS,
            "bound": "link" if moved / (LINK_GBS * 1e9) > mean_ms * 1e-3 else "gemm",
            "ms_per_step_unfused": mean_ms + g_ms + r_ms,
            "tflops": world * flops / (f_ms * 1e-3) / 1e12,
            "identical_to_nccl_gather": identical,
            "how": "epilogue TMA stores of each C tile to every rank's row-major buffer "
                   "(CUDA IPC) + one-word NCCL all-reduce per step",
        }
        del shards, full, go

    if rank != 0:
        return 0

    peaks = {}
    try:
        with open(os.path.join(ROOT, "MEASURED_PEAKS.json")) as f:
            peaks = json.load(f)
    except OSError:
        pass
    traffic = None
    tfile = os.path.join(ROOT, "profiles", "traffic.json")
    if os.path.exists(tfile):
        with open(tfile) as f:
            traffic = json.load(f).get(args.config)
    abytes = algorithmic_bytes(M, N, K, out_bytes, sparse)
    if M <= 128:
        # Decode shapes are HBM-bound: algorithmic bytes per launch / launch time against
        # the driver-measured copy bandwidth.
        hbm = peaks.get("hbm_gbs") or 6650.0
        ach = abytes / (mean_ms * 1e-3) / 1e9
        roofline = {"bound": "hbm", "achieved": ach, "peak": hbm, "unit": "GB/s",
                    "frac": ach / hbm,
                    "peak_source": "MEASURED_PEAKS.json hbm_gbs" if peaks.get("hbm_gbs")
                    else "fallback 6650 GB/s",
                    "traffic": traffic, "algorithmic_bytes": abytes,
                    "tcgen05_fp4_ladder": ladder}
    else:
        roofline = {"bound": "tensor", "achieved": achieved, "peak": peak_tf,
                    "unit": "TFLOP/s", "frac": achieved / peak_tf,
                    "peak_source": "tcgen05 kind::mxf4nvf4 ladder measured in this run "
                                   + ("(.sp M128 N256, 128 logical K per MMA, " if sparse else
                                      "(M128 N256 K64, ")
                                   + "on every SM, random E2M1 operands, best of 5 single "
                                     "launches)",
                    "tcgen05_fp4_ladder": ladder,
                    "bf16_measured_peak": peaks.get("bf16_tflops"),
                    "traffic": traffic, "algorithmic_bytes": abytes}
    cpu = None
    if world == 1 and not args.no_cpu_baseline:
        r = cpu_reference_sample(M, N, K, target_s=args.cpu_seconds)
        cpu = {"value": r["tflops"], "unit": "TFLOP/s", "cores": r["threads"], "kind": "port",
               "sample": f"{r['sample']}; {r['seconds']:.1f} s"}
    line = {
        "metric": "nvfp4_gemm_tflops", "value": value, "unit": "TFLOP/s", "n_gpus": world,
        "steps": args.steps, "warmup": args.warmup, "ms_per_step": mean_ms,
        "higher_is_better": True, "scaling": "strong" if strong else "weak", "vs_baseline": None,
        "dtype": "e2m1/ue4m3->f32",
        "data": "synthetic N(0,1), seeded, quantised on the GPU",
        "config": {"workload": desc, "M": M, "N_per_gpu": N, "N_total": n_total, "K": K, "out": od,
                   "parallelism": f"N-sharded x{world}" if world > 1 else "single GPU",
                   "l2": (f"weight rotated over {len(rot)} copies ({len(rot)} x "
                          f"{(B.packed.numel() + B.scales_tc.numel()) / 1e6:.1f} MB > 3x L2), "
                          "no flush; host enqueue ahead of a GPU spin; per-step CUDA events"
                          if decode else
                          "flushed (256 MiB write) before every step; per-step CUDA events"),
                   "tile_n": args.tile_n or "auto", "sf_layout": "tcgen05",
                   "step": (("quantise fp32 A fused into the GEMM (one launch)" if fused_qa else
                             "quantise fp32 A (GPU) + GEMM") if args.quantize_a else "GEMM")},
        "burst_tflops": burst_tf, "sustained_tflops": sust_tf,
        "roofline": roofline,
        "cpu_baseline": cpu,
        "e2e": {"value": world * flops / (e2e_ms * 1e-3) / 1e12, "unit": "TFLOP/s",
                "ms_per_step": e2e_ms, "h2d_bytes_per_step": int(h2d),
                "d2h_bytes_per_step": int(d2h)},
        "gpu_launches": args.steps * (2 if args.quantize_a and not fused_qa else 1),
        "clocks": clk,
    }
    if graph is not None:
        line["graph"] = graph
    if gather is not None:
        line["gather"] = gather
    if world == 1 and not args.no_extras:
        line["extra"] = run_extras(api, dev, args.extra_steps, ladder,
                                   peaks.get("hbm_gbs") or 6650.0, local_rank)
    print(json.dumps(line), flush=True)
    return 0


def main(argv=None):
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=20)
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--impl", default="b200", choices=["b200", "reference"])
    ap.add_argument("--config", default="c2", choices=sorted(CONFIGS))
    ap.add_argument("--tile-n", type=int, default=0)
    ap.add_argument("--cta-group", type=int, default=0,
                    help="0 = engine heuristic, 1 = one-SM tiles, 2 = SM-pair tiles")
    ap.add_argument("--cpu-seconds", type=float, default=12.0)
    ap.add_argument("--ref-step-s", type=float, default=3.0)
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--no-extras", action="store_true",
                    help="skip the other BASELINE configurations timed beside the headline (N=1)")
    ap.add_argument("--extra-steps", type=int, default=20)
    ap.add_argument("--quantize-a", action="store_true",
                    help="each step quantises fp32 A on the GPU before the GEMM (decode layers)")
    ap.add_argument("--b-static", action="store_true",
                    help="pass NVFP4_FLAG_B_STATIC (weights not written by the preceding launch) "
                         "so a decode GEMM streams its weight while the previous one finishes")
    ap.add_argument("--gather", action="store_true",
                    help="time the all-gather of the C column shards (N > 1; the default there): "
                         "NCCL after the GEMM, and fused into the GEMM's epilogue")
    ap.add_argument("--no-gather", action="store_true",
                    help="N > 1: time the weak-scaled GEMM only, without the all-gather legs")
    ap.add_argument("--kernel-only", action="store_true",
                    help="time the device steps only (no ladder, e2e, reference-style timing or "
                         "CPU baseline): the command profiled under ncu")
    args = ap.parse_args(argv)

    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local_rank = int(os.environ.get("LOCAL_RANK", "0"))
    if args.impl == "reference":
        return run_reference(args, rank, world)
    if world > 1:
        import torch
        import torch.distributed as dist
        torch.cuda.set_device(local_rank)
        dist.init_process_group("nccl", device_id=torch.device("cuda", local_rank))
    try:
        return run_b200(args, rank, world, local_rank)
    finally:
        if world > 1:
            import torch.distributed as dist
            dist.destroy_process_group()


if __name__ == "__main__":
    sys.exit(main())
