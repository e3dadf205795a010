// codec_dev.cuh - device restatement of the reference's scalar codecs (src/nvfp4.cu),
// shared by the codec kernels (codec.cu) and the GEMM epilogue that writes NVFP4 output
// (gemm_b200.cu), so that both produce the same bytes.
//   e2m1_quantize  :18-29  nearest of {0,.5,1,1.5,2,3,4,6}, ties to the smaller magnitude
//   e4m3_decode    :34-45  UE4M3, bias 7, subnormals; code 0x7F decodes to 480
//   e4m3_encode    :47-59  nearest code in 0..127, ties to the lower code, x clamped to 448
//   quantize       :62-97  per-block amax -> scale (amax/6)/g -> code -> x / (dec(code)*g)
#pragma once
#include <cstdint>

namespace nvfp4b200 {
namespace {

constexpr uint64_t kGolden = 0x9E3779B97F4A7C15ull;

__device__ __forceinline__ uint64_t splitmix_mix(uint64_t z) {
  z = (z ^ (z >> 30)) * 0xBF58476D1CE4E5B9ull;
  z = (z ^ (z >> 27)) * 0x94D049BB133111EBull;
  return z ^ (z >> 31);
}

// src/nvfp4.cu:34-45 for positive codes, built from the bit pattern (exact).
__device__ __forceinline__ float e4m3_decode_pos(int c) {
  const int e = (c >> 3) & 0xF, m = c & 7;
  if (e == 0) return __fmul_rn(static_cast<float>(m), 0.001953125f);  // m/8 * 2^-6
  return __int_as_float(((e + 120) << 23) | (m << 20));                 // (1+m/8) * 2^(e-7)
}
__device__ __forceinline__ float e4m3_decode_dev(uint8_t code) {
  const float v = e4m3_decode_pos(code & 0x7F);
  return (code & 0x80) ? -v : v;
}

// src/nvfp4.cu:47-59: the nearest code in 0..127 with ties to the lower code, computed from the
// float's bits. For x >= 2^-6, x = (1 + m/8 + r/2^23) * 2^E lies between code (E+7, m) and the
// next code up, 2^(E-3) apart; r > 2^19 is strictly nearer the upper one and r == 2^19 is a tie
// (both errors are exact float differences, the operands being within a factor of two). Below
// 2^-6 the codes are k/512 apart and x * 512 is exact. x is clamped to 448 (code 126) first, as
// in the reference; x <= 0 and NaN give 0.
__device__ __forceinline__ uint8_t e4m3_encode_dev(float x) {
  if (!(x > 0.0f)) return 0;
  if (448.0f < x) x = 448.0f;
  if (x >= 0.015625f) {
    const uint32_t b = __float_as_uint(x);
    const int e = static_cast<int>(b >> 23) - 127;  // -6 .. 8
    const uint32_t m = (b >> 20) & 7u, r = b & 0xFFFFFu;
    return static_cast<uint8_t>((((e + 7) << 3) | static_cast<int>(m)) + (r > 0x80000u ? 1 : 0));
  }
  const float f = __fmul_rn(x, 512.0f);
  const float k = floorf(f);
  return static_cast<uint8_t>(static_cast<int>(k) + (__fsub_rn(f, k) > 0.5f ? 1 : 0));
}

// src/nvfp4.cu:18-29: the nearest of {0,.5,1,1.5,2,3,4,6}, ties to the smaller magnitude,
// through float errors |a - mag| compared in order. Below 2^25 that is exactly the count of
// midpoints {.25,.75,1.25,1.75,2.5,3.5,5} strictly below |x| (checked against the reference's
// loop over all 2^32 floats); from 2^25 on, rounded errors tie and the loop's order decides, so
// it runs as written (infinities included). NaN gives 0 either way.
__device__ __forceinline__ uint8_t e2m1_quantize_dev(float x) {
  const uint8_t sign = (x < 0.0f) ? 0x8 : 0x0;
  const float a = fabsf(x);
  if (a < 33554432.0f) {
    const int i = (a > 0.25f) + (a > 0.75f) + (a > 1.25f) + (a > 1.75f) + (a > 2.5f) + (a > 3.5f) +
                  (a > 5.0f);
    return static_cast<uint8_t>(sign | i);
  }
  const float mag[8] = {0.0f, 0.5f, 1.0f, 1.5f, 2.0f, 3.0f, 4.0f, 6.0f};
  int best = 0;
  float best_err = fabsf(__fsub_rn(a, mag[0]));
#pragma unroll
  for (int i = 1; i < 8; ++i) {
    const float e = fabsf(__fsub_rn(a, mag[i]));
    if (e < best_err) { best_err = e; best = i; }
  }
  return static_cast<uint8_t>(sign | best);
}

// e2m1_quantize_dev(x / dec) without the division, for one scale block. With y = |x| / dec
// exact and every midpoint m having an even float mantissa, the rounded quotient exceeds m
// exactly when y > m + ulp(m)/2 (a tie rounds back to m), i.e. when |x| > (m + ulp(m)/2) * dec.
// That product is exact in double (25 + 24 significant bits), and for a float a and a double T,
// a > T exactly when a > T rounded down to float. So each block takes seven products and roundings
// and each element seven float compares. The quotient's sign bit survives unless it rounds to
// zero (|x| / dec <= 2^-150). Quotients from 2^24 up, NaN and infinities take the division path.
struct E2m1Thresholds {
  float t[7];   // rounded-down (m + ulp(m)/2) * dec for the midpoints .25 .. 5
  float big;    // rounded-up 2^24 * dec: the fast path needs |x| below it
  float zero;   // rounded-down 2^-150 * dec: quotients at or below it round to zero
};
__device__ __forceinline__ E2m1Thresholds e2m1_thresholds(float dec) {
  const double d = static_cast<double>(dec);
  E2m1Thresholds th;
  th.t[0] = __double2float_rd((0.25 + 0x1p-26) * d);
  th.t[1] = __double2float_rd((0.75 + 0x1p-25) * d);
  th.t[2] = __double2float_rd((1.25 + 0x1p-24) * d);
  th.t[3] = __double2float_rd((1.75 + 0x1p-24) * d);
  th.t[4] = __double2float_rd((2.5 + 0x1p-23) * d);
  th.t[5] = __double2float_rd((3.5 + 0x1p-23) * d);
  th.t[6] = __double2float_rd((5.0 + 0x1p-22) * d);
  th.big = __double2float_ru(16777216.0 * d);
  th.zero = __double2float_rd(0x1p-150 * d);
  return th;
}
// The fast path alone, for |x| < th.big (NaN included: its code is 0, as the division's).
__device__ __forceinline__ uint32_t e2m1_code_fast(float x, const E2m1Thresholds& th) {
  const float a = fabsf(x);
  // The count of thresholds below a, by binary search over the sorted thresholds.
  const bool h = a > th.t[3];
  const bool m = a > (h ? th.t[5] : th.t[1]);
  const bool l = a > (h ? (m ? th.t[6] : th.t[4]) : (m ? th.t[2] : th.t[0]));
  const uint32_t i = (h ? 4u : 0u) | (m ? 2u : 0u) | (l ? 1u : 0u);
  return ((x < 0.0f && a > th.zero) ? 0x8u : 0x0u) | i;
}
__device__ __forceinline__ uint8_t e2m1_quantize_scaled(float x, float dec, const E2m1Thresholds& th) {
  if (fabsf(x) < th.big) return static_cast<uint8_t>(e2m1_code_fast(x, th));
  return e2m1_quantize_dev(__fdiv_rn(x, dec));
}

// 8 consecutive codes of a block into one word (low nibble = first element). When the block's
// amax is below th.big every element takes the fast path (amax ignores NaN, which the fast path
// codes as 0), so the block branches once instead of once per element.
__device__ __forceinline__ uint32_t e2m1_pack8(const float* x, float dec, const E2m1Thresholds& th,
                                               bool fast) {
  uint32_t w = 0;
  if (fast) {
#pragma unroll
    for (int j = 0; j < 8; ++j) w |= e2m1_code_fast(x[j], th) << (4 * j);
  } else {
#pragma unroll
    for (int j = 0; j < 8; ++j) w |= static_cast<uint32_t>(e2m1_quantize_scaled(x[j], dec, th)) << (4 * j);
  }
  return w;
}

__device__ __forceinline__ float e2m1_decode_dev(uint8_t code) {
  const float mag[8] = {0.0f, 0.5f, 1.0f, 1.5f, 2.0f, 3.0f, 4.0f, 6.0f};
  const float m = mag[code & 7];
  return (code & 8) ? -m : m;
}

// One block of 16 values (src/nvfp4.cu:66-95): returns its scale code and writes 16 E2M1
// codes into two words (low nibble = even element).
__device__ __forceinline__ uint8_t quantize16_dev(const float (&x)[16], float g, uint32_t& lo, uint32_t& hi) {
  float amax = 0.0f;
#pragma unroll
  for (int j = 0; j < 16; ++j) {
    const float a = fabsf(x[j]);
    if (amax < a) amax = a;  // std::max(amax, a): NaN never replaces amax
  }
  const float scale = (amax > 0.0f) ? __fdiv_rn(__fdiv_rn(amax, 6.0f), g) : 1.0f;
  const uint8_t sc = e4m3_encode_dev(scale);
  float dec = __fmul_rn(e4m3_decode_dev(sc), g);
  if (dec <= 0.0f) dec = 1.0f;
  const E2m1Thresholds th = e2m1_thresholds(dec);
  const bool fast = amax < th.big;
  lo = e2m1_pack8(x, dec, th, fast);
  hi = e2m1_pack8(x + 8, dec, th, fast);
  return sc;
}

}  // namespace
}  // namespace nvfp4b200
