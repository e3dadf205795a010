// gemm_sparse.cu - 2:4 structured-sparse NVFP4 GEMM (GemmMode::Sparse).
//
// The reference has no data path for this mode (its backends refuse it,
// src/gemm_custom.cu:135-139, src/gemm_cutlass.cu:195-198). The tcgen05 .sp kernel is not
// built yet; the call reports that, following the reference's unsupported-mode convention.
#include <string>

#include "internal.h"

namespace nvfp4b200 {

bool gemm_sparse(const Nvfp4DeviceOperands&, cudaStream_t, std::string* err) {
  set_err(err, "2:4 sparse mode not supported by this build of the b200 backend yet");
  return false;
}

}  // namespace nvfp4b200
