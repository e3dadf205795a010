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
  lo = 0;
  hi = 0;
#pragma unroll
  for (int j = 0; j < 8; ++j) lo |= static_cast<uint32_t>(e2m1_quantize_dev(__fdiv_rn(x[j], dec))) << (4 * j);
#pragma unroll
  for (int j = 0; j < 8; ++j) hi |= static_cast<uint32_t>(e2m1_quantize_dev(__fdiv_rn(x[8 + j], dec))) << (4 * j);
  return sc;
}

}  // namespace
}  // namespace nvfp4b200
