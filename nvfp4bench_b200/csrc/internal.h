// internal.h - declarations shared by the engine's translation units (not installed).
#pragma once

#include <cstdint>
#include <string>

#include <cuda.h>
#include <cuda_runtime.h>

#include "gemm.h"

namespace nvfp4b200 {

inline void set_err(std::string* err, const std::string& msg) {
  if (err) *err = msg;
}

// ---- GEMM (gemm_b200.cu, gemm_decode.cu, gemm_noalloc.cu) ---------------------------------------------
size_t sf_tcgen05_bytes(int rows, int K);
bool gemm_dense(const Nvfp4DeviceOperands& op, cudaStream_t s, std::string* err);
// Dense GEMM with scales already in the tcgen05 layout; `out` is op.d or op.c.
bool gemm_dense_tc(const Nvfp4DeviceOperands& op, const uint8_t* sfa, const uint8_t* sfb,
                   void* out, cudaStream_t s, std::string* err);
// Canonical-scale dense GEMM that reorders into a fixed static scratch (gemm_noalloc.cu).
bool gemm_noalloc(const Nvfp4DeviceOperands& op, cudaStream_t s, std::string* err);
size_t noalloc_scratch_bytes();
bool gemm_sparse(const Nvfp4DeviceOperands& op, cudaStream_t s, std::string* err);
uint32_t* device_error_word(std::string* err);
// Tensor map of a packed FP4 operand [rows][K/2] (box 128 bytes x box_rows, 128-byte
// swizzle), from the engine's map cache.
bool operand_map(CUtensorMap* map, const void* base, int rows, int K, int box_rows,
                 std::string* err);
int device_sms(std::string* err);
// Compute capability major of the current device (0 on error, with *err set).
int device_cc_major(std::string* err);
// Weight-streaming GEMM for M <= 128 tokens (gemm_decode.cu); scales in the tcgen05 layout.
bool gemm_decode(const Nvfp4DeviceOperands& op, const uint8_t* sfa, const uint8_t* sfb,
                 void* out, cudaStream_t s, std::string* err);
// Decode GEMM with the quantisation of fp32 A fused in (gemm_decode.cu): A's packed values go
// to op.a_packed and its tcgen05 scales to sfa.
bool gemm_decode_quantize_a(const Nvfp4DeviceOperands& op, const float* a_src, uint8_t* sfa,
                            const uint8_t* sfb, void* out, cudaStream_t s, std::string* err);
bool wait_selftest(uint64_t limit_ns, std::string* err);

// ---- codecs (codec.cu) ---------------------------------------------------------------
bool fill_uniform(float* out, size_t n, uint64_t seed, cudaStream_t s, std::string* err);
bool fill_normal(float* out, size_t n, uint64_t seed, cudaStream_t s, std::string* err);
bool quantize(const float* src, int rows, int cols, float global_scale, uint8_t* packed,
              uint8_t* scales, uint8_t* scales_tc, cudaStream_t s, std::string* err);
bool dequantize(const uint8_t* packed, const uint8_t* scales, int rows, int cols,
                float global_scale, float* out, cudaStream_t s, std::string* err);
bool sf_to_tcgen05(const uint8_t* scales, int rows, int K, uint8_t* out, cudaStream_t s,
                   std::string* err);
// Both GEMM operands' canonical scales reordered in one launch (b may be null: a only).
bool sf_to_tcgen05_pair(const uint8_t* a, int rows_a, const uint8_t* b, int rows_b, int K,
                        uint8_t* out_a, uint8_t* out_b, cudaStream_t s, std::string* err);
// Block size 16 (NVFP4, the reference's codec) or 32 (the scale block of the sparse MMA); the
// tcgen05 scale layout of block 32 is the block-16 layout of a [rows x cols/2] operand.
bool quantize_block(const float* src, int rows, int cols, float global_scale, int block,
                    uint8_t* packed, uint8_t* scales, uint8_t* scales_tc, cudaStream_t s,
                    std::string* err);
bool dequantize_block(const uint8_t* packed, const uint8_t* scales, int rows, int cols,
                      float global_scale, int block, float* out, cudaStream_t s, std::string* err);
// Pair-wise 2:4 sparsity of A (the sparse kernel in gemm_b200.cu): metadata [rows][K/16], prune (fp32, in place),
// compress (packed [rows][K/2] -> values [rows][K/4]).
bool sparse_meta(int rows, int K, uint64_t seed, uint8_t* meta, cudaStream_t s, std::string* err);
bool sparse_prune(float* a, int rows, int K, const uint8_t* meta, cudaStream_t s, std::string* err);
bool sparse_compress(const uint8_t* packed, int rows, int K, const uint8_t* meta, uint8_t* values,
                     cudaStream_t s, std::string* err);
// GPU mirror of the reference's naive FP32 oracle (src/reference.cu:9-17) with B as N x K.
bool naive_gemm_nt(const float* A, const float* B, int M, int N, int K, float* C, cudaStream_t s,
                   std::string* err);

// ---- roofs (roofs.cu) ----------------------------------------------------------------
bool measure_bandwidth(int kind, const void* src, void* dst, const void* src2, size_t bytes,
                       int iters, double* gbs, cudaStream_t s, std::string* err);
// One rung of the tcgen05 FP4 ladder. cta_group 1: `units` CTAs of M=128 x N=n MMAs; 2: `units`
// SM pairs of M=256 x N=256. seed 0 stages zero operands, otherwise pseudo-random E2M1 bytes.
// sustained 0: best of `reps` launches timed one by one; 1: mean of `reps` back-to-back launches.
// sparse 1 (cta_group 1 only): tcgen05.mma.sp rungs, 128 logical K per MMA.
struct PeakOptions {
  int n, cta_group, units, iters, reps;
  uint32_t seed;
  int sustained;
  int sparse;
};
bool peak_ladder_ex(const PeakOptions& o, double* tflops, double* sm_mhz, cudaStream_t s,
                    std::string* err);
bool peak_ladder(int n, int ctas, int iters, int reps, double* tflops, cudaStream_t s,
                 std::string* err);
// SM-pair rung: `clusters` clusters of 2 CTAs, cta_group::2 MMAs of M=256 x n x K=64.
bool peak_ladder_pair(int n, int clusters, int iters, int reps, double* tflops, cudaStream_t s,
                      std::string* err);

}  // namespace nvfp4b200
