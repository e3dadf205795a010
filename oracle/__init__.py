"""ctypes bindings for the CPU oracle (oracle/liborc.so) and the reference build (oracle/_ref).

TEST INFRASTRUCTURE ONLY. This package is the checker for the CUDA product path. Only
tests/, __graft_entry__.smoke() and bench.py's cpu_baseline / ``--impl reference`` legs may
import it; nothing under nvfp4bench_b200/ does.

``liborc.so`` restates the reference's src/nvfp4.cu (codecs, packing, splitmix64 fill) and
src/reference.cu (naive FP32 GEMM, k ascending). ``_ref/libnvfp4ref.so`` is the reference's
own src/nvfp4.cu compiled unchanged (oracle/Makefile); it exists only where the reference
source tree was present at build time, and its .so travels with the repository snapshot.
"""
from __future__ import annotations

import ctypes as C
import os
import subprocess

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(HERE, "liborc.so")
REF_PATH = os.path.join(HERE, "_ref", "libnvfp4ref.so")

_u8p = C.POINTER(C.c_uint8)
_f32p = C.POINTER(C.c_float)
_i32p = C.POINTER(C.c_int)


def build() -> None:
    """Compile liborc.so, and _ref/ when the reference source tree can be found: the
    NVFP4BENCH_REF environment variable names the reference project root; unset, a checkout
    named ``reference`` beside this repository is used when it exists."""
    env = dict(os.environ)
    if not env.get("NVFP4BENCH_REF") and not env.get("REF_SRC"):
        sibling = os.path.join(os.path.dirname(os.path.dirname(HERE)), "reference")
        if os.path.isfile(os.path.join(sibling, "src", "nvfp4.cu")):
            env["NVFP4BENCH_REF"] = sibling
    subprocess.run(["make", "-s", "-C", HERE], check=True, env=env)


def _load(path: str):
    if not os.path.exists(path):
        build()
    return C.CDLL(path)


_lib = None
_ref = None


def lib():
    global _lib
    if _lib is None:
        _lib = _load(LIB_PATH)
        L = _lib
        L.orc_e2m1_decode.restype = C.c_float
        L.orc_e2m1_decode.argtypes = [C.c_uint8]
        L.orc_e2m1_quantize.restype = C.c_uint8
        L.orc_e2m1_quantize.argtypes = [C.c_float]
        L.orc_e4m3_decode.restype = C.c_float
        L.orc_e4m3_decode.argtypes = [C.c_uint8]
        L.orc_e4m3_encode.restype = C.c_uint8
        L.orc_e4m3_encode.argtypes = [C.c_float]
        L.orc_quantize.argtypes = [_f32p, C.c_int, C.c_int, C.c_float, _u8p, _u8p]
        L.orc_dequantize.argtypes = [_u8p, _u8p, C.c_int, C.c_int, C.c_float, _f32p]
        L.orc_make_uniform.argtypes = [C.c_int, C.c_int, C.c_uint64, _f32p]
        L.orc_gemm_nt.argtypes = [_f32p, _f32p, C.c_int, C.c_int, C.c_int, _f32p, C.c_int]
        L.orc_gemm_nt_rows.argtypes = [_f32p, _f32p, C.c_int, C.c_int, C.c_int, _i32p, C.c_int,
                                       _f32p, C.c_int]
        L.orc_max_rel_error.restype = C.c_double
        L.orc_max_rel_error.argtypes = [_f32p, _f32p, C.c_size_t]
        L.orc_sf_tcgen05_bytes.restype = C.c_size_t
        L.orc_sf_tcgen05_bytes.argtypes = [C.c_int, C.c_int]
        L.orc_sf_to_tcgen05.argtypes = [_u8p, C.c_int, C.c_int, _u8p]
        L.orc_quantize_block.argtypes = [_f32p, C.c_int, C.c_int, C.c_float, C.c_int, _u8p, _u8p]
        L.orc_dequantize_block.argtypes = [_u8p, _u8p, C.c_int, C.c_int, C.c_float, C.c_int, _f32p]
        L.orc_sparse_meta.argtypes = [C.c_int, C.c_int, C.c_uint64, _u8p]
        L.orc_sparse_prune.argtypes = [_f32p, C.c_int, C.c_int, _u8p]
        L.orc_sparse_compress.argtypes = [_u8p, C.c_int, C.c_int, _u8p, _u8p]
        L.orc_default_threads.restype = C.c_int
    return _lib


def ref_available() -> bool:
    return os.path.exists(REF_PATH)


def ref():
    """The reference's own nvfp4.cu (compiled from its source tree)."""
    global _ref
    if _ref is None:
        if not ref_available():
            raise FileNotFoundError(REF_PATH)
        _ref = C.CDLL(REF_PATH)
        R = _ref
        R.ref_e2m1_quantize.restype = C.c_uint8
        R.ref_e2m1_quantize.argtypes = [C.c_float]
        R.ref_e2m1_decode.restype = C.c_float
        R.ref_e2m1_decode.argtypes = [C.c_uint8]
        R.ref_e4m3_encode.restype = C.c_uint8
        R.ref_e4m3_encode.argtypes = [C.c_float]
        R.ref_e4m3_decode.restype = C.c_float
        R.ref_e4m3_decode.argtypes = [C.c_uint8]
        R.ref_quantize.argtypes = [_f32p, C.c_int, C.c_int, C.c_float, _u8p, _u8p]
        R.ref_dequantize.argtypes = [_u8p, _u8p, C.c_int, C.c_int, C.c_float, _f32p]
        R.ref_make_random.argtypes = [C.c_int, C.c_int, C.c_uint64, _f32p]
    return _ref


def _p(a: np.ndarray, t):
    assert a.flags["C_CONTIGUOUS"]
    return a.ctypes.data_as(t)


# ---- numpy-level helpers -------------------------------------------------------------
def quantize(x: np.ndarray, global_scale: float = 1.0, use_ref: bool = False):
    """fp32 [rows, cols] -> (packed uint8 [rows, cols/2], scales uint8 [rows, cols/16])."""
    x = np.ascontiguousarray(x, dtype=np.float32)
    rows, cols = x.shape
    packed = np.empty((rows, cols // 2), np.uint8)
    scales = np.empty((rows, cols // 16), np.uint8)
    fn = ref().ref_quantize if use_ref else lib().orc_quantize
    fn(_p(x, _f32p), rows, cols, global_scale, _p(packed, _u8p), _p(scales, _u8p))
    return packed, scales


def dequantize(packed: np.ndarray, scales: np.ndarray, cols: int, global_scale: float = 1.0,
               use_ref: bool = False) -> np.ndarray:
    packed = np.ascontiguousarray(packed, dtype=np.uint8)
    scales = np.ascontiguousarray(scales, dtype=np.uint8)
    rows = packed.shape[0]
    out = np.empty((rows, cols), np.float32)
    fn = ref().ref_dequantize if use_ref else lib().orc_dequantize
    fn(_p(packed, _u8p), _p(scales, _u8p), rows, cols, global_scale, _p(out, _f32p))
    return out


def make_uniform(rows: int, cols: int, seed: int, use_ref: bool = False) -> np.ndarray:
    out = np.empty((rows, cols), np.float32)
    fn = ref().ref_make_random if use_ref else lib().orc_make_uniform
    fn(rows, cols, seed, _p(out, _f32p))
    return out


def gemm_nt(A: np.ndarray, B: np.ndarray, threads: int = 0) -> np.ndarray:
    """C = A @ B.T, naive FP32, k ascending (src/reference.cu:9-17)."""
    A = np.ascontiguousarray(A, dtype=np.float32)
    B = np.ascontiguousarray(B, dtype=np.float32)
    M, K = A.shape
    N = B.shape[0]
    C_ = np.empty((M, N), np.float32)
    lib().orc_gemm_nt(_p(A, _f32p), _p(B, _f32p), M, N, K, _p(C_, _f32p), threads)
    return C_


def gemm_nt_rows(A: np.ndarray, B: np.ndarray, rows, threads: int = 0) -> np.ndarray:
    A = np.ascontiguousarray(A, dtype=np.float32)
    B = np.ascontiguousarray(B, dtype=np.float32)
    M, K = A.shape
    N = B.shape[0]
    r = np.ascontiguousarray(np.asarray(rows, dtype=np.int32))
    out = np.empty((len(r), N), np.float32)
    lib().orc_gemm_nt_rows(_p(A, _f32p), _p(B, _f32p), M, N, K, _p(r, _i32p), len(r),
                           _p(out, _f32p), threads)
    return out


def sf_to_tcgen05(scales: np.ndarray, K: int) -> np.ndarray:
    scales = np.ascontiguousarray(scales, dtype=np.uint8)
    rows = scales.shape[0]
    n = lib().orc_sf_tcgen05_bytes(rows, K)
    out = np.empty(n, np.uint8)
    lib().orc_sf_to_tcgen05(_p(scales, _u8p), rows, K, _p(out, _u8p))
    return out


def quantize_block(x: np.ndarray, block: int, global_scale: float = 1.0):
    """quantize() with `block` elements per scale: (packed [rows, cols/2], scales [rows, cols/block])."""
    x = np.ascontiguousarray(x, dtype=np.float32)
    rows, cols = x.shape
    packed = np.empty((rows, cols // 2), np.uint8)
    scales = np.empty((rows, cols // block), np.uint8)
    lib().orc_quantize_block(_p(x, _f32p), rows, cols, global_scale, block, _p(packed, _u8p),
                             _p(scales, _u8p))
    return packed, scales


def dequantize_block(packed: np.ndarray, scales: np.ndarray, cols: int, block: int,
                     global_scale: float = 1.0) -> np.ndarray:
    packed = np.ascontiguousarray(packed, dtype=np.uint8)
    scales = np.ascontiguousarray(scales, dtype=np.uint8)
    rows = packed.shape[0]
    out = np.empty((rows, cols), np.float32)
    lib().orc_dequantize_block(_p(packed, _u8p), _p(scales, _u8p), rows, cols, global_scale, block,
                               _p(out, _f32p))
    return out


def sparse_meta(rows: int, K: int, seed: int) -> np.ndarray:
    """Pair-wise 2:4 metadata [rows, K/16] (one nibble per group of 8 K elements)."""
    out = np.empty((rows, K // 16), np.uint8)
    lib().orc_sparse_meta(rows, K, seed, _p(out, _u8p))
    return out


def sparse_prune(a: np.ndarray, meta: np.ndarray) -> np.ndarray:
    a = np.array(a, dtype=np.float32, copy=True, order="C")
    meta = np.ascontiguousarray(meta, dtype=np.uint8)
    rows, K = a.shape
    lib().orc_sparse_prune(_p(a, _f32p), rows, K, _p(meta, _u8p))
    return a


def sparse_compress(packed: np.ndarray, meta: np.ndarray, K: int) -> np.ndarray:
    packed = np.ascontiguousarray(packed, dtype=np.uint8)
    meta = np.ascontiguousarray(meta, dtype=np.uint8)
    rows = packed.shape[0]
    out = np.empty((rows, K // 4), np.uint8)
    lib().orc_sparse_compress(_p(packed, _u8p), rows, K, _p(meta, _u8p), _p(out, _u8p))
    return out


def max_abs_error(got: np.ndarray, ref_: np.ndarray):
    """(max |got-ref|, max |ref|) in float64."""
    g = np.asarray(got, dtype=np.float64)
    r = np.asarray(ref_, dtype=np.float64)
    d = np.abs(g - r)
    me = float(np.nanmax(d)) if d.size else 0.0
    if np.isnan(d).any():
        me = float("inf")
    return me, float(np.abs(r).max()) if r.size else 0.0


def max_rel_error(got: np.ndarray, ref_: np.ndarray) -> float:
    g = np.ascontiguousarray(got, dtype=np.float32).ravel()
    r = np.ascontiguousarray(ref_, dtype=np.float32).ravel()
    return float(lib().orc_max_rel_error(_p(g, _f32p), _p(r, _f32p), g.size))


def default_threads() -> int:
    return int(lib().orc_default_threads())
