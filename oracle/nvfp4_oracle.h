/* nvfp4_oracle.h - CPU restatement of the reference's NVFP4 codecs and FP32 GEMM oracle.
 *
 * TEST INFRASTRUCTURE ONLY. This library is the checker for the CUDA product path
 * (nvfp4bench_b200/csrc). Only tests/, __graft_entry__.smoke() and bench.py's
 * cpu_baseline / --impl reference legs may load it. Nothing in the product links it.
 *
 * Parity pin: the codec functions are checked byte-for-byte against the reference's own
 * src/nvfp4.cu, compiled unchanged from its source tree into oracle/_ref/ (recipe in
 * oracle/Makefile), and against the golden fixtures in tests/golden/ that the same build
 * produced. The GEMM follows src/reference.cu:9-17 (naive FP32, k ascending).
 */
#ifndef NVFP4_ORACLE_H
#define NVFP4_ORACLE_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

/* src/nvfp4.cu:13-16 */
float orc_e2m1_decode(uint8_t code);
/* src/nvfp4.cu:18-29 - nearest magnitude, ties to the smaller one, NaN -> 0 */
uint8_t orc_e2m1_quantize(float x);
/* src/nvfp4.cu:34-45 */
float orc_e4m3_decode(uint8_t code);
/* src/nvfp4.cu:47-59 - linear nearest search over codes 0..127, ties to the lower code */
uint8_t orc_e4m3_encode(float x);

/* src/nvfp4.cu:62-97. Row-major fp32 [rows x cols] -> packed [rows x cols/2] (low nibble =
 * even column) and scales [rows x cols/16] (one e4m3 byte per 16 contiguous columns). */
void orc_quantize(const float* src, int rows, int cols, float global_scale,
                  uint8_t* packed, uint8_t* scales);
/* src/nvfp4.cu:99-112 */
void orc_dequantize(const uint8_t* packed, const uint8_t* scales, int rows, int cols,
                    float global_scale, float* out);
/* orc_quantize / orc_dequantize with `block` elements per scale (16 or 32; cols % block == 0). */
void orc_quantize_block(const float* src, int rows, int cols, float global_scale, int block,
                        uint8_t* packed, uint8_t* scales);
void orc_dequantize_block(const uint8_t* packed, const uint8_t* scales, int rows, int cols,
                          float global_scale, int block, float* out);
/* src/nvfp4.cu:115-129 - splitmix64 -> uniform [-1,1) */
void orc_make_uniform(int rows, int cols, uint64_t seed, float* out);

/* src/reference.cu:9-17 with B stored N x K (K contiguous):
 *   C[m][n] = sum_{k ascending} A[m][k] * B[n][k], one fp32 accumulator, no FMA contraction.
 * Rows are split over `threads` host threads (0 = one per online core). */
void orc_gemm_nt(const float* A, const float* B, int M, int N, int K, float* C, int threads);
/* Same as orc_gemm_nt for a subset of output rows: C_rows[i][n] for m = rows[i]. */
void orc_gemm_nt_rows(const float* A, const float* B, int M, int N, int K,
                      const int* rows, int nrows, float* C_rows, int threads);

/* Number of online host cores (the default thread count above). */
int orc_default_threads(void);

/* src/reference.cu:45-56 */
double orc_max_rel_error(const float* got, const float* ref, size_t n);
/* max |got - ref| and max |ref| (the engine's pass criterion is max|err| <= 1e-3 * max|ref|) */
void orc_max_abs_error(const float* got, const float* ref, size_t n, double* max_err,
                       double* max_ref);

/* Canonical scales [rows x K/16] -> the tcgen05 scale-factor layout used by the engine:
 * 512-byte atoms of 128 rows x 4 scales; atom (r/128, s/4) at ((r/128)*ceil(K/64) + s/4)*512,
 * byte (r%32)*16 + ((r/32)%4)*4 + s%4 inside it. Rows are padded to a multiple of 128 and
 * scale columns to a multiple of 4 with zero bytes. Returns the byte size written. */
size_t orc_sf_tcgen05_bytes(int rows, int K);
void orc_sf_to_tcgen05(const uint8_t* scales, int rows, int K, uint8_t* out);


/* Pair-wise 2:4 sparsity (the pattern of the tcgen05 .sp kind::mxf4nvf4 MMA on B200): per
 * group of 8 K elements (4 pairs) 2 pairs are kept; meta[rows*K/16] holds one nibble per
 * group (first kept pair | second << 2; even group in the low nibble). K % 16 == 0. */
void orc_sparse_meta(int rows, int K, uint64_t seed, uint8_t* meta);
void orc_sparse_prune(float* a, int rows, int K, const uint8_t* meta);
/* packed [rows][K/2] -> values [rows][K/4] (the kept pair bytes of each group, in order). */
void orc_sparse_compress(const uint8_t* packed, int rows, int K, const uint8_t* meta, uint8_t* values);

#ifdef __cplusplus
}
#endif
#endif
