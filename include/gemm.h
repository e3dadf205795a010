// gemm.h - launch interface of the NVFP4 GEMM backends (drop-in for the reference's
// src/gemm.h:13-40).
//
// D = A * B^T with NVFP4 operands: E2M1 values packed two per byte (low nibble = even
// index), one UE4M3 scale per 16 contiguous K elements, and one FP32 global scale per
// tensor. FP32 accumulation.
//
// Layouts (the reference's own text at src/gemm.h:10-11 says B is K x N, but its CUTLASS
// and custom backends and all of its benchmark configurations use N x K; this engine uses
// N x K throughout):
//   A packed [M][K/2], B packed [N][K/2].
//   Scales, SfLayout::Canonical: [rows][K/16] row-major (src/nvfp4.h:28-38).
//   Scales, SfLayout::Tcgen05:  512-byte atoms of 128 rows x 4 scales, atom (r/128, s/4)
//     at ((r/128)*ceil(K/64) + s/4)*512, byte (r%32)*16 + ((r/32)%4)*4 + s%4 inside it,
//     rows padded to 128 (see nvfp4_b200_sf_tcgen05_bytes). This is the order in which the
//     tensor cores read scales from Tensor Memory, so no reshuffle is needed per call.
//   Output: M x N row-major, FP32 into `c` (reference field) or, when `d` is set, the
//     type `out_dtype` into `d`.
//   2:4 sparse A (GemmMode::Sparse), the pair-wise form the tcgen05 .sp MMA executes: each
//     group of 8 consecutive K elements is 4 element pairs of which 2 are kept. a_packed
//     holds the kept values [M][K/4] (one byte = one kept pair, in order), a_meta [M][K/16]
//     one nibble per group (first kept pair | second << 2, even group in the low nibble).
//     A and B scales are one UE4M3 per 32 logical K elements (block 32, not 16): canonical
//     [rows][K/32], or the tcgen05 layout of nvfp4_b200_sf_tcgen05_bytes(rows, K / 2).
#pragma once

#include <string>

#include <cuda_runtime.h>

#include "common.h"

enum class SfLayout { Canonical = 0, Tcgen05 = 1 };
enum class OutDType { F32 = 0, BF16 = 1, NVFP4 = 2 };

// src/gemm.h:13-23, extended with defaulted fields (a reference-style initialisation of
// the first ten fields keeps its meaning).
struct Nvfp4DeviceOperands {
  const uint8_t* a_packed = nullptr;
  const uint8_t* a_scales = nullptr;
  float a_global = 1.0f;
  const uint8_t* b_packed = nullptr;
  const uint8_t* b_scales = nullptr;
  float b_global = 1.0f;
  float* c = nullptr;
  int M = 0, N = 0, K = 0;
  GemmMode mode = GemmMode::Dense;
  // ---- engine extensions --------------------------------------------------------------
  SfLayout sf_layout = SfLayout::Canonical;
  OutDType out_dtype = OutDType::F32;
  void* d = nullptr;                 // output of out_dtype; when null, `c` (FP32) is used
  const uint8_t* a_meta = nullptr;   // 2:4 metadata (GemmMode::Sparse)
  int cta_group = 0;                 // 0 = heuristic, 1 = one-SM tiles, 2 = SM-pair tiles
  int tile_n = 0;                    // 0 = heuristic, else 128 or 256 (one-SM dense tiles)
  // NVFP4 output (out_dtype NVFP4): `d` = packed [M][N/2], `d_scales` in d_sf_layout, quantised
  // exactly as quantize_to_nvfp4 (src/nvfp4.cu:62-97) with global scale d_global.
  uint8_t* d_scales = nullptr;
  float d_global = 1.0f;
  SfLayout d_sf_layout = SfLayout::Canonical;
  // The caller guarantees that B and its scales are not written by the work enqueued just
  // before this call on the stream: the decode kernel may then start streaming the weight
  // before that work completes (programmatic dependent launch).
  bool b_static = false;
  // Row pitch of `d` in elements (0 = N): `d` may be a column slice of a wider matrix.
  int ldd = 0;
  // Further destinations of every FP32/BF16 output tile, each addressed like `d` (same row
  // pitch): typically other GPUs' buffers mapped into this process, so that a column-sharded
  // GEMM's all-gather of C is done by the epilogue as the tiles complete. At most 7.
  void* const* d_peers = nullptr;
  int n_peers = 0;
};

// src/gemm.h:25-29. Each backend returns true on success; on failure it sets *err (which
// may be null) and returns false. Launches are asynchronous on `s`; nothing synchronises.
bool launch_gemm_stub(const Nvfp4DeviceOperands& op, cudaStream_t s, std::string* err);
bool launch_gemm_cutlass(const Nvfp4DeviceOperands& op, cudaStream_t s, std::string* err);
bool launch_gemm_custom(const Nvfp4DeviceOperands& op, cudaStream_t s, std::string* err);
// The B200 backend: hand-written sm_100a tcgen05 kernels (nvfp4bench_b200/csrc/gemm_b200.cu).
bool launch_gemm_b200(const Nvfp4DeviceOperands& op, cudaStream_t s, std::string* err);

// src/gemm.h:31-40
inline bool launch_gemm(KernelKind kind, const Nvfp4DeviceOperands& op, cudaStream_t s,
                        std::string* err) {
  switch (kind) {
    case KernelKind::Stub: return launch_gemm_stub(op, s, err);
    case KernelKind::Cutlass: return launch_gemm_cutlass(op, s, err);
    case KernelKind::Custom: return launch_gemm_custom(op, s, err);
    case KernelKind::B200: return launch_gemm_b200(op, s, err);
  }
  if (err) *err = "unknown kernel kind";
  return false;
}
