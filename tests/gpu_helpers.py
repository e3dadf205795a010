"""Shared helpers for the GPU parity tests: operands made on the GPU, checked on the CPU oracle."""
import numpy as np
import torch

TOL = 1e-3  # GEMM criterion: max |err| <= TOL * max |C_ref| (FP32 output)


def make_operand(api, rows, K, seed, dist="normal", global_scale=1.0):
    if dist == "normal":
        x = api.fill_normal(rows, K, seed)
    else:
        x = api.fill_uniform(rows, K, seed)
    t = api.quantize(x, global_scale)
    return x, t


def oracle_dequant(orc, t):
    p = t.packed.cpu().numpy()
    s = t.scales.cpu().numpy()
    return orc.dequantize(p, s, t.cols, t.global_scale)


def bf16_half_ulp(ref):
    """Half a bf16 ulp of |ref| (the rounding of a correct value to bf16)."""
    a = np.abs(ref).astype(np.float32)
    e = np.floor(np.log2(np.maximum(a, np.float32(2.0 ** -126))))
    return np.float32(2.0) ** (e - 8)


def check_gemm(got, ref, bf16=False, tol=TOL):
    got = np.asarray(got, np.float64)
    ref = np.asarray(ref, np.float64)
    cinf = np.abs(ref).max()
    err = np.abs(got - ref)
    bound = tol * cinf + (bf16_half_ulp(ref) if bf16 else 0.0)
    worst = float((err - bound).max())
    assert np.isfinite(got).all(), "non-finite output"
    assert worst <= 0, f"max|err|={err.max():.3e} cinf={cinf:.3e} (bound {tol}*cinf{' + bf16 half-ulp' if bf16 else ''})"
    return float(err.max() / max(cinf, 1e-30))


def run_gemm(api, a, b, M, N, K, out_dtype=torch.float32, sf_layout=None, **kw):
    sf_layout = api.SF_TCGEN05 if sf_layout is None else sf_layout
    out = torch.empty((M, N), dtype=out_dtype, device="cuda")
    if sf_layout == api.SF_TCGEN05:
        sa, sb = a.scales_tc, b.scales_tc
    else:
        sa, sb = a.scales, b.scales
    api.gemm(a.packed, sa, b.packed, sb, M, N, K, out, a_global=a.global_scale,
             b_global=b.global_scale, sf_layout=sf_layout, **kw)
    torch.cuda.synchronize()
    assert api.device_error() == 0
    return out
