"""Generate the golden fixtures in tests/golden/ from the reference's own host codecs.

Run where the reference source tree exists (it builds oracle/_ref/libnvfp4ref.so from the
reference's src/nvfp4.cu, unchanged):  python tests/golden/make_golden.py

Fixtures:
  codec_kat.json  e2m1_quantize / e4m3_encode / e4m3_decode / e2m1_decode outputs of the
                  reference for hand-picked inputs (ties, clamps, NaN, inf, subnormals) and
                  for seeded random inputs.
  quant_small.npz make_random_matrix(16, 256, 1234) and (16, 256, 1234^0xABCDEF), their
                  quantize_to_nvfp4 packed bytes and scales, and dequantize_nvfp4 outputs;
                  plus an N(0,1)*3 matrix (seed 7, numpy) with its reference quantisation.
  int_gemm.npz    the exact-integer GEMM known answer of the reference's self-check
                  (src/gemm_warp_mxf4.cu:124-157): codes 0..7 from its LCG with seeds
                  0x111 / 0x222, unit scales; expected C = A*B in exact integer arithmetic.
"""
import json
import os
import sys

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, os.path.dirname(os.path.dirname(HERE)))
import oracle  # noqa: E402

E2M1_INPUTS = [0.0, -0.0, 0.25, 0.2499999, 0.2500001, 0.75, 1.25, 1.75, 2.5, 3.5, 5.0, 7.0,
               -0.75, -1.75, -5.0, 6.0, 6.5, 100.0, -100.0, 1e-30, 1e30,
               float("nan"), float("inf"), float("-inf")]
E4M3_INPUTS = [1.0 / 6.0, 0.15, 1e-4, 500.0, 448.0, 447.9, 449.0, 0.0, -1.0,
               2.0 ** -9, 2.0 ** -10, 3 * 2.0 ** -11, 0.0009765625, 0.001953125, 0.015625,
               0.0146484375, 1.0, 1.0625, 1.0624999, 1.0625001, 240.0, 232.0, 248.0,
               float("nan"), float("inf")]


def lcg_codes(n, seed):
    """src/gemm_warp_mxf4.cu:124-125."""
    s = seed
    out = np.empty(n, np.uint8)
    for i in range(n):
        s = (s * 6364136223846793005 + 1) & 0xFFFFFFFFFFFFFFFF
        out[i] = (s >> 33) % 8
    return out


def main():
    oracle.build()
    R = oracle.ref()
    rng = np.random.default_rng(20261201)
    rnd = np.concatenate([rng.standard_normal(2000) * 4, rng.uniform(0, 500, 2000),
                          np.exp(rng.uniform(-14, 6.5, 2000))]).astype(np.float32)
    kat = {
        "e2m1_quantize": [[float(x), int(R.ref_e2m1_quantize(x))] for x in E2M1_INPUTS],
        "e4m3_encode": [[float(x), int(R.ref_e4m3_encode(x))] for x in E4M3_INPUTS],
        "e4m3_decode": [float(R.ref_e4m3_decode(c)) for c in range(256)],
        "e2m1_decode": [float(R.ref_e2m1_decode(c)) for c in range(16)],
        "random_inputs_f32_hex": [np.float32(x).view(np.uint32).item() for x in rnd],
        "random_e2m1": [int(R.ref_e2m1_quantize(float(x))) for x in rnd],
        "random_e4m3": [int(R.ref_e4m3_encode(float(abs(x)))) for x in rnd],
        "uniform_seed1234_first8": [float(v) for v in oracle.make_uniform(1, 8, 1234, use_ref=True)[0]],
    }
    with open(os.path.join(HERE, "codec_kat.json"), "w") as f:
        json.dump(kat, f, indent=0)

    a = oracle.make_uniform(16, 256, 1234, use_ref=True)
    b = oracle.make_uniform(16, 256, 1234 ^ 0xABCDEF, use_ref=True)
    n = (np.random.default_rng(7).standard_normal((16, 256)) * 3).astype(np.float32)
    n[0, :16] = 0.0                      # an all-zero block (scale 1.0 branch)
    n[1, 5] = np.float32(np.nan)         # NaN is ignored by amax and quantises to 0
    n[2, 7] = np.float32(1e6)            # scale clamps to 448
    out = {"a": a, "b": b, "n": n}
    for name, x in (("a", a), ("b", b), ("n", n)):
        p, s = oracle.quantize(x, use_ref=True)
        out[name + "_packed"], out[name + "_scales"] = p, s
        out[name + "_dq"] = oracle.dequantize(p, s, x.shape[1], use_ref=True)
    p, s = oracle.quantize(n, 0.5, use_ref=True)
    out["n_g05_packed"], out["n_g05_scales"] = p, s
    np.savez_compressed(os.path.join(HERE, "quant_small.npz"), **out)

    M = N = K = 128
    ca = lcg_codes(M * K, 0x111).reshape(M, K)
    cb = lcg_codes(K * N, 0x222).reshape(K, N)
    mag = np.array([0, .5, 1, 1.5, 2, 3, 4, 6], np.float64)
    c_exact = mag[ca] @ mag[cb]
    np.savez_compressed(os.path.join(HERE, "int_gemm.npz"), codes_a=ca, codes_b_kn=cb,
                        c=c_exact.astype(np.float32))
    print("wrote fixtures to", HERE)


if __name__ == "__main__":
    main()
