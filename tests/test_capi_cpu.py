"""CPU: the C-ABI library loads and exports exactly what include/nvfp4_b200.h declares."""
import ctypes as C
import os
import re

import pytest
import torch

from nvfp4bench_b200 import api, build

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


@pytest.fixture(scope="module")
def lib():
    if not os.path.exists(build.LIB):
        build.build()
    return api.lib()


def declared_symbols():
    names = set()
    inc = os.path.join(ROOT, "include")
    for f in os.listdir(inc):
        if not f.endswith(".h"):
            continue
        text = open(os.path.join(inc, f)).read()
        if 'extern "C"' not in text:
            continue
        names |= set(re.findall(r"\b(nvfp4_b200_\w+)\s*\(", text))
    return names


def test_exports_every_declared_symbol(lib):
    decl = declared_symbols()
    assert decl, "no C-ABI declarations found"
    assert decl == set(api.EXPORTED), decl ^ set(api.EXPORTED)
    for name in decl:
        assert hasattr(lib, name), name


def test_version_and_sizes(lib):
    assert "sm_100a" in api.version()
    assert api.sf_tcgen05_bytes(4096, 4096) == 32 * 64 * 512
    assert api.sf_tcgen05_bytes(1, 16) == 512
    assert api.sf_tcgen05_bytes(0, 64) == 0


def test_null_args_rejected_without_gpu(lib):
    buf = C.create_string_buffer(256)
    rc = lib.nvfp4_b200_gemm(None, None, buf, 256)
    assert rc == 1 and b"null" in buf.value


def test_bad_mode_rejected_without_gpu(lib):
    args = api.GemmArgs()
    args.mode = 7
    buf = C.create_string_buffer(256)
    assert lib.nvfp4_b200_gemm(C.byref(args), None, buf, 256) == 1
    assert b"mode" in buf.value


def test_reference_backend_slots_report_not_built():
    """The C++ interface keeps the reference's KernelKind values (src/common.h:33)."""
    text = open(os.path.join(ROOT, "include", "gemm.h")).read()
    for k in ("Stub", "Cutlass", "Custom", "B200"):
        assert f"KernelKind::{k}" in text


def test_every_export_declares_argtypes():
    """Each entry point with arguments has ctypes argtypes (an untyped 64-bit argument that
    lands in a stack slot is passed as 32 bits)."""
    from nvfp4bench_b200 import api
    L = api.lib()
    for name in api.EXPORTED:
        fn = getattr(L, name)
        if name in ("nvfp4_b200_version",):
            continue
        assert fn.argtypes is not None, name


def test_gemm_args_pitch_and_peers_without_gpu(lib):
    """A column slice gets its row stride as ldc; peers travel as a C array of addresses."""
    wide = torch.empty((8, 640), dtype=torch.bfloat16)
    out = wide[:, 128:384]
    args = api.gemm_args(None, None, None, None, 8, 256, 64, out, peers=[0x1000, 0x2000])
    assert args.ldc == 640 and args.n_peers == 2
    assert [args.c_peers[i] for i in range(2)] == [0x1000, 0x2000]
    plain = api.gemm_args(None, None, None, None, 8, 640, 64, wide)
    assert plain.ldc == 0 and plain.n_peers == 0 and not plain.c_peers


def test_ipc_argument_errors_without_gpu(lib):
    buf = C.create_string_buffer(256)
    off = C.c_size_t(0)
    assert lib.nvfp4_b200_ipc_handle(None, None, C.byref(off), buf, 256) == 1
    assert lib.nvfp4_b200_ipc_close(C.c_void_p(0x1234), buf, 256) == 1
    assert b"not returned" in buf.value


def test_pitch_and_peer_argument_errors_without_gpu(lib):
    buf = C.create_string_buffer(256)
    out = torch.empty((8, 256), dtype=torch.bfloat16)
    args = api.gemm_args(None, None, None, None, 8, 256, 64, out)
    args.ldc = 128
    assert lib.nvfp4_b200_gemm(C.byref(args), None, buf, 256) == 1 and b"ldc" in buf.value
    args = api.gemm_args(None, None, None, None, 8, 256, 64, out, peers=[0x1000] * 8)
    assert lib.nvfp4_b200_gemm(C.byref(args), None, buf, 256) == 1 and b"n_peers" in buf.value
    args = api.gemm_args(None, None, None, None, 8, 256, 64, out)
    args.n_peers = 2  # no array
    assert lib.nvfp4_b200_gemm(C.byref(args), None, buf, 256) == 1 and b"n_peers" in buf.value


def test_noalloc_refuses_nvfp4_output_without_gpu(lib):
    args = api.GemmArgs()
    args.mode = api.MODE_DENSE
    args.sf_layout = api.SF_CANONICAL
    args.out_dtype = api.OUT_NVFP4
    buf = C.create_string_buffer(256)
    assert lib.nvfp4_b200_gemm_noalloc(C.byref(args), None, buf, 256) == 3
    assert b"NVFP4 output is not supported" in buf.value
