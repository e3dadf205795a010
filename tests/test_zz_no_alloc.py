"""GPU: the allocation-free GEMM entry point (nvfp4_b200_gemm_noalloc) through the C ABI.

Callers such as CUDA-graph capture, servers that own all device memory through their own
pool, or latency-critical loops cannot let a library cudaMalloc a workspace. This entry point
reorders the canonical scales into a fixed scratch array compiled into the library instead.
The test checks its output against the regular entry point (nvfp4_b200_gemm, canonical
scales) on consecutive calls (each later call reuses the scratch the previous one left
behind). Both entry points run the same kernel on the same bytes, so the outputs must be
bit-identical, not merely within the suite's GEMM tolerance. One shape has M <= 128, which
routes through the weight-streaming decode kernel. A problem too large for the scratch and
NVFP4 output are refused.
This file is collected last so that a run stopping at the first failure has run all others.
"""
import ctypes as C

import numpy as np
import pytest
import torch

from gpu_helpers import TOL, make_operand

pytestmark = pytest.mark.gpu


def _args(api, a, b, M, N, K, out):
    return api.GemmArgs(a.packed.data_ptr(), a.scales.data_ptr(), a.global_scale,
                        b.packed.data_ptr(), b.scales.data_ptr(), b.global_scale,
                        out.data_ptr(), M, N, K, api.MODE_DENSE, api.SF_CANONICAL,
                        api.OUT_BF16 if out.dtype == torch.bfloat16 else api.OUT_F32,
                        None, 0, 0)


def _call(fn, args):
    err = C.create_string_buffer(512)
    rc = fn(C.byref(args), C.c_void_p(torch.cuda.current_stream().cuda_stream), err, 512)
    return rc, err.value.decode()


@pytest.mark.parametrize("out_dtype", [torch.float32, torch.bfloat16])
def test_noalloc_matches_regular_entry_point(api, out_dtype):
    L = api.lib()
    # Consecutive calls with different shapes; the third (M <= 128) takes the decode kernel.
    shapes = [(512, 768, 1024, 5), (300, 520, 288, 6), (64, 768, 1024, 7), (64, 768, 1024, 8)]
    for M, N, K, seed in shapes:
        _, a = make_operand(api, M, K, seed, global_scale=0.5)
        _, b = make_operand(api, N, K, seed + 100, global_scale=2.0)
        ref = torch.empty((M, N), dtype=out_dtype, device="cuda")
        got = torch.full((M, N), float("nan"), dtype=out_dtype, device="cuda")
        rc, msg = _call(L.nvfp4_b200_gemm, _args(api, a, b, M, N, K, ref))
        assert rc == 0, msg
        rc, msg = _call(L.nvfp4_b200_gemm_noalloc, _args(api, a, b, M, N, K, got))
        assert rc == 0, msg
        torch.cuda.synchronize()
        r = ref.float().cpu().numpy().astype(np.float64)
        g = got.float().cpu().numpy().astype(np.float64)
        assert np.isfinite(g).all()
        assert np.abs(g - r).max() <= TOL * np.abs(r).max()
        assert torch.equal(got, ref), f"{M}x{N}x{K}: no-alloc output differs from nvfp4_b200_gemm"
    assert api.device_error() == 0


def test_noalloc_refuses_nvfp4_output(api):
    L = api.lib()
    dummy = torch.empty(16, dtype=torch.uint8, device="cuda")
    args = api.GemmArgs(dummy.data_ptr(), dummy.data_ptr(), 1.0, dummy.data_ptr(),
                        dummy.data_ptr(), 1.0, dummy.data_ptr(), 128, 128, 128, api.MODE_DENSE,
                        api.SF_CANONICAL, api.OUT_NVFP4, None, 0, 0)
    rc, msg = _call(L.nvfp4_b200_gemm_noalloc, args)
    assert rc == 3 and "NVFP4 output is not supported" in msg


def test_noalloc_rejects_oversized_problem(api):
    L = api.lib()
    cap = int(L.nvfp4_b200_gemm_noalloc_scratch_bytes())
    assert cap == 16 << 20
    # (M + N) * K / 16 bytes of reordered scales: 8192 + 8192 rows at K = 32768 need 32 MiB,
    # more than the scratch holds. No operand memory is touched before the size check.
    M = N = 8192
    K = 32768
    dummy = torch.empty(16, dtype=torch.uint8, device="cuda")
    args = api.GemmArgs(dummy.data_ptr(), dummy.data_ptr(), 1.0, dummy.data_ptr(),
                        dummy.data_ptr(), 1.0, dummy.data_ptr(), M, N, K, api.MODE_DENSE,
                        api.SF_CANONICAL, api.OUT_F32, None, 0, 0)
    rc, msg = _call(L.nvfp4_b200_gemm_noalloc, args)
    assert rc == 1 and "too large" in msg
