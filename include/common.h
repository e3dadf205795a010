// common.h - shared types of the NVFP4 GEMM engine's C++ interface.
//
// Mirrors the reference's src/common.h:33-77 (KernelKind, GemmMode, GemmProblem,
// to_string, gemm_flops, BenchResult) so that a backend written against the reference's
// interface compiles unchanged; KernelKind gains the B200 value (the tcgen05 backend).
#pragma once

#include <cstdint>
#include <cstdio>
#include <cstdlib>
#include <string>
#include <vector>

#include <cuda_runtime.h>

// src/common.h:13-21 - harness-side CUDA error check (exits; backends never use it).
#define CHECK_CUDA(call)                                                              \
  do {                                                                                \
    cudaError_t _e = (call);                                                          \
    if (_e != cudaSuccess) {                                                          \
      std::fprintf(stderr, "[CUDA error] %s:%d: %s (%s)\n", __FILE__, __LINE__,        \
                   cudaGetErrorString(_e), #call);                                    \
      std::exit(EXIT_FAILURE);                                                        \
    }                                                                                 \
  } while (0)

// src/common.h:23-30 - the harness's non-fatal variant (warns and continues).
#define CHECK_CUDA_NOEXIT(call)                                                       \
  do {                                                                                \
    cudaError_t _e = (call);                                                          \
    if (_e != cudaSuccess) {                                                          \
      std::fprintf(stderr, "[CUDA warn] %s:%d: %s (%s)\n", __FILE__, __LINE__,         \
                   cudaGetErrorString(_e), #call);                                    \
    }                                                                                 \
  } while (0)

// src/common.h:33. Stub/Cutlass/Custom are the reference's GB10 backends; this engine
// implements only B200 and reports the others as not built.
enum class KernelKind { Stub, Cutlass, Custom, B200 };
// src/common.h:34. Sparse == 2:4 structured sparsity on A.
enum class GemmMode { Dense, Sparse };

// src/common.h:36-41
struct GemmProblem {
  int m = 8192;
  int n = 8192;
  int k = 8192;
  GemmMode mode = GemmMode::Dense;
};

// src/common.h:43-53
inline const char* to_string(KernelKind k) {
  switch (k) {
    case KernelKind::Stub: return "stub";
    case KernelKind::Cutlass: return "cutlass";
    case KernelKind::Custom: return "custom";
    case KernelKind::B200: return "b200";
  }
  return "?";
}
inline const char* to_string(GemmMode m) { return m == GemmMode::Dense ? "dense" : "2:4"; }

// src/common.h:55-60. Dense and 2:4 sparse count the same logical FLOPs.
inline double gemm_flops(const GemmProblem& p) {
  return 2.0 * double(p.m) * double(p.n) * double(p.k);
}

// src/common.h:63-77, plus the engine's roofline columns.
struct BenchResult {
  GemmProblem problem;
  KernelKind kernel = KernelKind::B200;
  double median_ms = 0.0;
  double min_ms = 0.0;
  double tflops = 0.0;        // sustained, from the median time
  double peak_tflops = 0.0;   // burst, from the min time
  double pct_dense_peak = 0.0;
  double pct_sparse_peak = 0.0;
  bool validated = false;
  bool valid_pass = false;
  double max_rel_err = 0.0;
  double max_abs_err_over_cinf = 0.0;  // engine criterion: <= 1e-3
  double algorithmic_bytes = 0.0;
  double gbs = 0.0;                    // algorithmic bytes / min time
  bool ok = false;
  std::string note;
};
