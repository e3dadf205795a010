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

__device__ __forceinline__ uint8_t e4m3_encode_dev(float x) {
  if (!(x > 0.0f)) return 0;  // x <= 0 -> 0; NaN -> 0 (no error ever compares smaller)
  if (448.0f < x) x = 448.0f;
  int lo = 1, hi = 126;       // dec(0) = 0 < x and dec(126) = 448 >= x
  while (lo < hi) {
    const int mid = (lo + hi) >> 1;
    if (e4m3_decode_pos(mid) >= x) hi = mid; else lo = mid + 1;
  }
  const float eh = fabsf(__fsub_rn(e4m3_decode_pos(hi), x));
  const float el = fabsf(__fsub_rn(e4m3_decode_pos(hi - 1), x));
  return static_cast<uint8_t>(eh < el ? hi : hi - 1);
}

// src/nvfp4.cu:18-29, verbatim in structure.
__device__ __forceinline__ uint8_t e2m1_quantize_dev(float x) {
  const float mag[8] = {0.0f, 0.5f, 1.0f, 1.5f, 2.0f, 3.0f, 4.0f, 6.0f};
  const uint8_t sign = (x < 0.0f) ? 0x8 : 0x0;
  const float a = fabsf(x);
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
