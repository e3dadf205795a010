"""ctypes binding of the engine's C ABI (include/nvfp4_b200.h) plus torch-tensor helpers.

This is the binding a Python user of the reference's hot path would write against the
C ABI; torch supplies device memory and streams only. The library is loaded from the
package's lib/ directory (built in-tree by ``python -m nvfp4bench_b200.build``); when it is
missing every call raises - there is no CPU fallback.
"""
from __future__ import annotations

import ctypes as C
import os
from dataclasses import dataclass
from typing import Optional

import torch

from . import build as _build

# NVFP4_B200_LIB overrides the library path (to compare two builds side by side).
LIB_PATH = os.environ.get("NVFP4_B200_LIB", _build.LIB)

MODE_DENSE, MODE_SPARSE24 = 0, 1
SF_CANONICAL, SF_TCGEN05 = 0, 1
OUT_F32, OUT_BF16, OUT_NVFP4 = 0, 1, 2
FLAG_B_STATIC = 1

# Every symbol include/nvfp4_b200.h declares (checked by the CPU tests).
EXPORTED = [
    "nvfp4_b200_gemm", "nvfp4_b200_quantize", "nvfp4_b200_dequantize",
    "nvfp4_b200_fill_uniform", "nvfp4_b200_fill_normal", "nvfp4_b200_sf_tcgen05_bytes",
    "nvfp4_b200_sf_to_tcgen05", "nvfp4_b200_measure_bandwidth", "nvfp4_b200_peak",
    "nvfp4_b200_device_error", "nvfp4_b200_wait_selftest", "nvfp4_b200_version",
    "nvfp4_b200_gemm_noalloc", "nvfp4_b200_gemm_noalloc_scratch_bytes", "nvfp4_b200_peak_ex",
    "nvfp4_b200_quantize_ex", "nvfp4_b200_dequantize_ex", "nvfp4_b200_sparse_meta",
    "nvfp4_b200_sparse_prune", "nvfp4_b200_sparse_compress", "nvfp4_b200_ipc_handle",
    "nvfp4_b200_ipc_open", "nvfp4_b200_ipc_close", "nvfp4_b200_gemm_quantize_a",
]
IPC_HANDLE_BYTES = 64


class Nvfp4Error(RuntimeError):
    """A nonzero return code of the C ABI, with its message."""

    def __init__(self, code: int, msg: str):
        super().__init__(f"[nvfp4_b200 error {code}] {msg}")
        self.code = code


class GemmArgs(C.Structure):
    """Nvfp4GemmArgs (include/nvfp4_b200.h)."""

    _fields_ = [
        ("a_packed", C.c_void_p), ("a_scales", C.c_void_p), ("a_global", C.c_float),
        ("b_packed", C.c_void_p), ("b_scales", C.c_void_p), ("b_global", C.c_float),
        ("c", C.c_void_p), ("M", C.c_int), ("N", C.c_int), ("K", C.c_int),
        ("mode", C.c_int), ("sf_layout", C.c_int), ("out_dtype", C.c_int),
        ("a_meta", C.c_void_p), ("cta_group", C.c_int), ("tile_n", C.c_int),
        ("c_scales", C.c_void_p), ("c_global", C.c_float), ("c_sf_layout", C.c_int),
        ("flags", C.c_int), ("ldc", C.c_int), ("c_peers", C.POINTER(C.c_void_p)),
        ("n_peers", C.c_int),
    ]


_lib = None


def lib():
    """Load libnvfp4_b200.so (raises if it has not been built)."""
    global _lib
    if _lib is None:
        if not os.path.exists(LIB_PATH):
            raise FileNotFoundError(
                f"{LIB_PATH} is missing; build it with `python -m nvfp4bench_b200.build`")
        L = C.CDLL(LIB_PATH)
        vp, sz, ip = C.c_void_p, C.c_size_t, C.c_int
        errs = [C.c_char_p, sz]
        L.nvfp4_b200_gemm.argtypes = [C.POINTER(GemmArgs), vp, *errs]
        L.nvfp4_b200_gemm_noalloc.argtypes = [C.POINTER(GemmArgs), vp, *errs]
        L.nvfp4_b200_gemm_quantize_a.argtypes = [C.POINTER(GemmArgs), vp, vp, *errs]
        L.nvfp4_b200_gemm_noalloc_scratch_bytes.argtypes = []
        L.nvfp4_b200_gemm_noalloc_scratch_bytes.restype = sz
        L.nvfp4_b200_quantize.argtypes = [vp, ip, ip, C.c_float, vp, vp, vp, vp, *errs]
        L.nvfp4_b200_dequantize.argtypes = [vp, vp, ip, ip, C.c_float, vp, vp, *errs]
        L.nvfp4_b200_quantize_ex.argtypes = [vp, ip, ip, C.c_float, ip, vp, vp, vp, vp, *errs]
        L.nvfp4_b200_dequantize_ex.argtypes = [vp, vp, ip, ip, C.c_float, ip, vp, vp, *errs]
        L.nvfp4_b200_sparse_meta.argtypes = [ip, ip, C.c_uint64, vp, vp, *errs]
        L.nvfp4_b200_sparse_prune.argtypes = [vp, ip, ip, vp, vp, *errs]
        L.nvfp4_b200_sparse_compress.argtypes = [vp, ip, ip, vp, vp, vp, *errs]
        L.nvfp4_b200_fill_uniform.argtypes = [vp, ip, ip, C.c_uint64, vp, *errs]
        L.nvfp4_b200_fill_normal.argtypes = [vp, ip, ip, C.c_uint64, vp, *errs]
        L.nvfp4_b200_sf_tcgen05_bytes.argtypes = [ip, ip]
        L.nvfp4_b200_sf_tcgen05_bytes.restype = sz
        L.nvfp4_b200_sf_to_tcgen05.argtypes = [vp, ip, ip, vp, vp, *errs]
        L.nvfp4_b200_measure_bandwidth.argtypes = [ip, vp, vp, vp, sz, ip,
                                                   C.POINTER(C.c_double), vp, *errs]
        L.nvfp4_b200_peak.argtypes = [ip, ip, ip, ip, C.POINTER(C.c_double), vp, *errs]
        L.nvfp4_b200_peak_ex.argtypes = [ip, ip, ip, ip, ip, C.c_uint32, ip, ip,
                                         C.POINTER(C.c_double), C.POINTER(C.c_double), vp, *errs]
        L.nvfp4_b200_device_error.argtypes = [ip, C.POINTER(C.c_uint32), *errs]
        L.nvfp4_b200_wait_selftest.argtypes = [C.c_uint64, C.POINTER(C.c_uint32), *errs]
        L.nvfp4_b200_ipc_handle.argtypes = [vp, vp, C.POINTER(sz), *errs]
        L.nvfp4_b200_ipc_open.argtypes = [vp, sz, C.POINTER(vp), *errs]
        L.nvfp4_b200_ipc_close.argtypes = [vp, *errs]
        L.nvfp4_b200_version.restype = C.c_char_p
        for name in EXPORTED:
            if name not in ("nvfp4_b200_sf_tcgen05_bytes", "nvfp4_b200_version",
                            "nvfp4_b200_gemm_noalloc_scratch_bytes"):
                getattr(L, name).restype = C.c_int
        _lib = L
    return _lib


def _call(fn, *args):
    buf = C.create_string_buffer(512)
    rc = fn(*args, buf, C.c_size_t(len(buf)))
    if rc != 0:
        raise Nvfp4Error(rc, buf.value.decode(errors="replace"))


def _stream(stream) -> C.c_void_p:
    # A typed pointer: a bare Python int is passed as a 32-bit value, which in a stack-passed
    # argument slot leaves the upper half of the 64-bit handle undefined.
    if stream is None:
        return C.c_void_p(torch.cuda.current_stream().cuda_stream)
    if isinstance(stream, torch.cuda.Stream):
        return C.c_void_p(stream.cuda_stream)
    return C.c_void_p(int(stream))


def _ptr(t: Optional[torch.Tensor]):
    return None if t is None else t.data_ptr()


# ---- entry points -------------------------------------------------------------------------
def _out_kind(out, out_scales):
    if out.dtype == torch.float32:
        return OUT_F32
    if out.dtype == torch.bfloat16:
        return OUT_BF16
    if out.dtype == torch.uint8 and out_scales is not None:
        return OUT_NVFP4
    raise ValueError("out must be float32, bfloat16, or uint8 packed NVFP4 with out_scales")


def gemm(a_packed, a_scales, b_packed, b_scales, M: int, N: int, K: int, out: torch.Tensor,
         a_global: float = 1.0, b_global: float = 1.0, sf_layout: int = SF_TCGEN05,
         mode: int = MODE_DENSE, a_meta=None, cta_group: int = 0, tile_n: int = 0,
         out_scales=None, out_global: float = 1.0, out_sf_layout: int = SF_CANONICAL,
         peers=None, stream=None) -> torch.Tensor:
    """D = (a_global*b_global) * A @ B^T into `out`: float32 or bfloat16 [M, N] (a column slice
    of a wider row-major matrix is fine: its row stride is the pitch), or packed NVFP4 uint8
    [M, N/2] with `out_scales` (canonical [M, N/16] or tcgen05 layout) and `out_global`.
    `peers`: device addresses (ints) of further destinations that receive every tile, each
    addressed like `out` with the same pitch (the fused all-gather; see shard.GatheredOutput)."""
    args = gemm_args(a_packed, a_scales, b_packed, b_scales, M, N, K, out, a_global=a_global,
                     b_global=b_global, sf_layout=sf_layout, mode=mode, a_meta=a_meta,
                     cta_group=cta_group, tile_n=tile_n, out_scales=out_scales,
                     out_global=out_global, out_sf_layout=out_sf_layout, peers=peers)
    _call(lib().nvfp4_b200_gemm, C.byref(args), _stream(stream))
    return out


def gemm_args(a_packed, a_scales, b_packed, b_scales, M, N, K, out, **kw) -> GemmArgs:
    """Prebuilt argument block for repeated launches (see launch())."""
    od = _out_kind(out, kw.get("out_scales"))
    ldc = 0
    if od != OUT_NVFP4 and out.dim() == 2 and out.stride(1) == 1 and out.stride(0) != N:
        ldc = out.stride(0)
    peers = list(kw.get("peers") or [])
    arr = (C.c_void_p * max(1, len(peers)))(*peers)
    args = GemmArgs(_ptr(a_packed), _ptr(a_scales), kw.get("a_global", 1.0), _ptr(b_packed),
                    _ptr(b_scales), kw.get("b_global", 1.0), _ptr(out), M, N, K,
                    kw.get("mode", MODE_DENSE), kw.get("sf_layout", SF_TCGEN05), od,
                    _ptr(kw.get("a_meta")), kw.get("cta_group", 0), kw.get("tile_n", 0),
                    _ptr(kw.get("out_scales")), kw.get("out_global", 1.0),
                    kw.get("out_sf_layout", SF_CANONICAL),
                    FLAG_B_STATIC if kw.get("b_static") else 0, ldc,
                    C.cast(arr, C.POINTER(C.c_void_p)) if peers else None, len(peers))
    args._peers_keepalive = arr  # the C array must outlive every launch of these arguments
    return args


def launch(args: GemmArgs, stream=None) -> None:
    _call(lib().nvfp4_b200_gemm, C.byref(args), _stream(stream))


def launch_quantize_a(args: GemmArgs, a_src: torch.Tensor, stream=None) -> None:
    """nvfp4_b200_gemm_quantize_a: quantise fp32 `a_src` [M, K] into args' A buffers (packed and
    tcgen05 scales, both outputs) and run the GEMM, fused into one launch for decode shapes."""
    if a_src.dtype != torch.float32 or not a_src.is_contiguous():
        raise ValueError("a_src must be a contiguous float32 tensor")
    _call(lib().nvfp4_b200_gemm_quantize_a, C.byref(args), C.c_void_p(a_src.data_ptr()),
          _stream(stream))


def ipc_handle(t: torch.Tensor):
    """(handle bytes, offset) exporting the device allocation that holds `t`'s first byte."""
    h = C.create_string_buffer(IPC_HANDLE_BYTES)
    off = C.c_size_t(0)
    _call(lib().nvfp4_b200_ipc_handle, C.c_void_p(t.data_ptr()), h, C.byref(off))
    return h.raw, off.value


def ipc_open(handle: bytes, offset: int) -> int:
    """This process's device address of the byte another process exported (see ipc_handle)."""
    assert len(handle) == IPC_HANDLE_BYTES
    p = C.c_void_p(0)
    _call(lib().nvfp4_b200_ipc_open, C.c_char_p(handle), C.c_size_t(offset), C.byref(p))
    return int(p.value)


def ipc_close(ptr: int) -> None:
    _call(lib().nvfp4_b200_ipc_close, C.c_void_p(ptr))


def sf_tcgen05_bytes(rows: int, K: int) -> int:
    return int(lib().nvfp4_b200_sf_tcgen05_bytes(rows, K))


@dataclass
class Nvfp4Tensor:
    """Device NVFP4 tensor (the reference's Nvfp4Tensor, src/nvfp4.h:28-38, on the GPU)."""

    rows: int
    cols: int
    global_scale: float
    packed: torch.Tensor             # uint8 [rows, cols/2]
    scales: Optional[torch.Tensor]   # uint8 [rows, cols/16] canonical
    scales_tc: Optional[torch.Tensor]  # uint8 [sf_tcgen05_bytes] tcgen05 layout


def quantize(x: torch.Tensor, global_scale: float = 1.0, canonical: bool = True,
             tcgen05: bool = True, stream=None) -> Nvfp4Tensor:
    """GPU quantize_to_nvfp4 (byte-identical to src/nvfp4.cu:62-97)."""
    assert x.is_cuda and x.dtype == torch.float32 and x.is_contiguous() and x.dim() == 2
    rows, cols = x.shape
    packed = torch.empty((rows, cols // 2), dtype=torch.uint8, device=x.device)
    sc = torch.empty((rows, cols // 16), dtype=torch.uint8, device=x.device) if canonical else None
    tc = torch.empty(sf_tcgen05_bytes(rows, cols), dtype=torch.uint8, device=x.device) \
        if tcgen05 else None
    _call(lib().nvfp4_b200_quantize, x.data_ptr(), rows, cols, global_scale, packed.data_ptr(),
          _ptr(sc), _ptr(tc), _stream(stream))
    return Nvfp4Tensor(rows, cols, global_scale, packed, sc, tc)


def dequantize(t: Nvfp4Tensor, stream=None) -> torch.Tensor:
    out = torch.empty((t.rows, t.cols), dtype=torch.float32, device=t.packed.device)
    _call(lib().nvfp4_b200_dequantize, t.packed.data_ptr(), t.scales.data_ptr(), t.rows, t.cols,
          t.global_scale, out.data_ptr(), _stream(stream))
    return out


def quantize_block(x: torch.Tensor, block: int, global_scale: float = 1.0, canonical: bool = True,
                   tcgen05: bool = True, stream=None) -> Nvfp4Tensor:
    """quantize() with `block` (16 or 32) elements per scale; block 32 is the scale block of the
    sparse MMA (scales [rows, cols/32]; tcgen05 layout of a [rows, cols/2] block-16 operand)."""
    assert x.is_cuda and x.dtype == torch.float32 and x.is_contiguous() and x.dim() == 2
    rows, cols = x.shape
    packed = torch.empty((rows, cols // 2), dtype=torch.uint8, device=x.device)
    sc = torch.empty((rows, cols // block), dtype=torch.uint8, device=x.device) if canonical else None
    vcols = cols if block == 16 else cols // 2
    tc = torch.empty(sf_tcgen05_bytes(rows, vcols), dtype=torch.uint8, device=x.device) \
        if tcgen05 else None
    _call(lib().nvfp4_b200_quantize_ex, x.data_ptr(), rows, cols, global_scale, block,
          packed.data_ptr(), _ptr(sc), _ptr(tc), _stream(stream))
    return Nvfp4Tensor(rows, cols, global_scale, packed, sc, tc)


def dequantize_block(t: Nvfp4Tensor, block: int, stream=None) -> torch.Tensor:
    out = torch.empty((t.rows, t.cols), dtype=torch.float32, device=t.packed.device)
    _call(lib().nvfp4_b200_dequantize_ex, t.packed.data_ptr(), t.scales.data_ptr(), t.rows, t.cols,
          t.global_scale, block, out.data_ptr(), _stream(stream))
    return out


def sparse_meta(rows: int, K: int, seed: int, device="cuda", stream=None) -> torch.Tensor:
    """Pair-wise 2:4 metadata uint8 [rows, K/16] (see nvfp4_b200_sparse_meta)."""
    out = torch.empty((rows, K // 16), dtype=torch.uint8, device=device)
    _call(lib().nvfp4_b200_sparse_meta, rows, K, C.c_uint64(seed), out.data_ptr(), _stream(stream))
    return out


def sparse_prune(a: torch.Tensor, meta: torch.Tensor, stream=None) -> torch.Tensor:
    """Zero the dropped pairs of fp32 [rows, K] in place; returns `a`."""
    rows, K = a.shape
    _call(lib().nvfp4_b200_sparse_prune, a.data_ptr(), rows, K, meta.data_ptr(), _stream(stream))
    return a


def sparse_compress(packed: torch.Tensor, meta: torch.Tensor, K: int, stream=None) -> torch.Tensor:
    """packed [rows, K/2] -> kept values [rows, K/4]."""
    rows = packed.shape[0]
    out = torch.empty((rows, K // 4), dtype=torch.uint8, device=packed.device)
    _call(lib().nvfp4_b200_sparse_compress, packed.data_ptr(), rows, K, meta.data_ptr(),
          out.data_ptr(), _stream(stream))
    return out


def fill_uniform(rows: int, cols: int, seed: int, device="cuda", stream=None) -> torch.Tensor:
    out = torch.empty((rows, cols), dtype=torch.float32, device=device)
    _call(lib().nvfp4_b200_fill_uniform, out.data_ptr(), rows, cols, seed, _stream(stream))
    return out


def fill_normal(rows: int, cols: int, seed: int, device="cuda", stream=None) -> torch.Tensor:
    out = torch.empty((rows, cols), dtype=torch.float32, device=device)
    _call(lib().nvfp4_b200_fill_normal, out.data_ptr(), rows, cols, seed, _stream(stream))
    return out


def sf_to_tcgen05(scales: torch.Tensor, rows: int, K: int, stream=None) -> torch.Tensor:
    out = torch.empty(sf_tcgen05_bytes(rows, K), dtype=torch.uint8, device=scales.device)
    _call(lib().nvfp4_b200_sf_to_tcgen05, scales.data_ptr(), rows, K, out.data_ptr(),
          _stream(stream))
    return out


def measure_bandwidth(kind: int, src: torch.Tensor, dst: Optional[torch.Tensor],
                      src2: Optional[torch.Tensor], nbytes: int, iters: int = 10,
                      stream=None) -> float:
    g = C.c_double(0.0)
    _call(lib().nvfp4_b200_measure_bandwidth, kind, src.data_ptr(), _ptr(dst), _ptr(src2), nbytes,
          iters, C.byref(g), _stream(stream))
    return g.value


def peak(n: int = 256, ctas: int = 148, iters: int = 4096, reps: int = 5, stream=None) -> float:
    t = C.c_double(0.0)
    _call(lib().nvfp4_b200_peak, n, ctas, iters, reps, C.byref(t), _stream(stream))
    return t.value


def peak_ex(n: int = 256, cta_group: int = 1, units: int = 148, iters: int = 4096, reps: int = 5,
            seed: int = 0, sustained: bool = False, sparse: bool = False, stream=None) -> tuple:
    """(TFLOP/s, SM MHz of CTA 0) of one ladder rung; see nvfp4_b200_peak_ex."""
    t = C.c_double(0.0)
    mhz = C.c_double(0.0)
    _call(lib().nvfp4_b200_peak_ex, n, cta_group, units, iters, reps, C.c_uint32(seed),
          1 if sustained else 0, 1 if sparse else 0, C.byref(t), C.byref(mhz), _stream(stream))
    return t.value, mhz.value


def device_error(clear: bool = True) -> int:
    w = C.c_uint32(0)
    _call(lib().nvfp4_b200_device_error, 1 if clear else 0, C.byref(w))
    return int(w.value)


def wait_selftest(limit_ns: int = 20_000_000) -> int:
    w = C.c_uint32(0)
    _call(lib().nvfp4_b200_wait_selftest, limit_ns, C.byref(w))
    return int(w.value)


def version() -> str:
    return lib().nvfp4_b200_version().decode()
