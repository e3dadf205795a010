// ref_shim.cpp - C entry points over the reference's own host codecs (src/nvfp4.cu),
// which this recipe compiles unchanged from the reference source tree.
//
// TEST INFRASTRUCTURE ONLY: used by tests/ and tests/golden/make_golden.py to pin the
// oracle restatement (nvfp4_oracle.c) against the reference itself. The resulting
// library lives in oracle/_ref/ and is never linked into the product.
#include <cstring>
#include <vector>
#include "nvfp4.h"  // reference header: src/nvfp4.h

extern "C" {

uint8_t ref_e2m1_quantize(float x) { return e2m1_quantize(x); }
float ref_e2m1_decode(uint8_t c) { return e2m1_decode(c); }
uint8_t ref_e4m3_encode(float x) { return e4m3_encode(x); }
float ref_e4m3_decode(uint8_t c) { return e4m3_decode(c); }

// src/nvfp4.h:40-42 quantize_to_nvfp4, flattened into caller-owned buffers.
void ref_quantize(const float* src, int rows, int cols, float global_scale,
                  uint8_t* packed, uint8_t* scales) {
  std::vector<float> v(src, src + size_t(rows) * cols);
  Nvfp4Tensor t = quantize_to_nvfp4(v, rows, cols, global_scale);
  std::memcpy(packed, t.packed.data(), t.packed.size());
  std::memcpy(scales, t.scales.data(), t.scales.size());
}

// src/nvfp4.h:44-45 dequantize_nvfp4.
void ref_dequantize(const uint8_t* packed, const uint8_t* scales, int rows, int cols,
                    float global_scale, float* out) {
  Nvfp4Tensor t;
  t.rows = rows; t.cols = cols; t.global_scale = global_scale;
  t.packed.assign(packed, packed + size_t(rows) * (cols / 2));
  t.scales.assign(scales, scales + size_t(rows) * (cols / 16));
  std::vector<float> o = dequantize_nvfp4(t);
  std::memcpy(out, o.data(), o.size() * sizeof(float));
}

// src/nvfp4.h:47-48 make_random_matrix.
void ref_make_random(int rows, int cols, uint64_t seed, float* out) {
  std::vector<float> v = make_random_matrix(rows, cols, seed);
  std::memcpy(out, v.data(), v.size() * sizeof(float));
}

}  // extern "C"
