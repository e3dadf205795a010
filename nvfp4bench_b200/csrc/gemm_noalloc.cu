// gemm_noalloc.cu - the GEMM for callers that must not allocate device memory.
//
// nvfp4_b200_gemm with canonical [rows][K/16] scales reorders both operands' scales into the
// tensor-core layout first, in a workspace it grows with cudaMalloc. Some callers cannot let
// a library allocate: code running inside CUDA-graph capture (an allocation there breaks or
// invalidates the capture), inference servers that carve all device memory into their own
// pool up front and forbid later allocations, and real-time loops where a cudaMalloc's
// implicit device synchronisation would stall the stream. nvfp4_b200_gemm_noalloc serves
// them: the reorder goes into a fixed scratch array that lives in this library's device
// image, so no call allocates or frees anything.
//
// The scratch is a file-scope __device__ array of kNoAllocScratchBytes (16 MiB), held by
// every GPU that loads the library until the process exits. Host code cannot pass the
// array's name to a kernel (on the host it is only a stand-in symbol); set-up therefore
// asks the runtime for its device address with cudaGetSymbolAddress, once per device with
// that device current, on the first call made on that device. Make that first call before
// any stream capture. All calls share the one array and leave the previous call's bytes in
// it (the reorder rewrites every byte it later reads, padding included). Each GPU has its own
// copy, but two calls on the same GPU whose work overlaps (for example on two streams) race
// on it: serialise them.
#include <cuda_runtime.h>

#include <mutex>
#include <string>
#include <vector>

#include "gemm.h"
#include "internal.h"

namespace nvfp4b200 {
namespace {

constexpr size_t kNoAllocScratchBytes = size_t(16) << 20;

static __device__ __align__(256) uint8_t g_noalloc_scratch[kNoAllocScratchBytes];

std::mutex g_na_mu;
std::vector<uint8_t*> g_na_ptr;  // per device: device address of g_noalloc_scratch

uint8_t* scratch_for_current_device(std::string* err) {
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess) {
    set_err(err, "cudaGetDevice failed");
    return nullptr;
  }
  std::lock_guard<std::mutex> lk(g_na_mu);
  if (static_cast<int>(g_na_ptr.size()) <= dev) g_na_ptr.resize(dev + 1, nullptr);
  if (!g_na_ptr[dev]) {
    void* ptr = nullptr;
    cudaError_t e = cudaGetSymbolAddress(&ptr, g_noalloc_scratch);
    if (e != cudaSuccess || !ptr) {
      set_err(err, std::string("cudaGetSymbolAddress of the no-alloc scratch failed: ") +
                       cudaGetErrorString(e));
      return nullptr;
    }
    g_na_ptr[dev] = static_cast<uint8_t*>(ptr);
  }
  return g_na_ptr[dev];
}

size_t round256(size_t n) { return (n + 255) & ~size_t(255); }

}  // namespace

size_t noalloc_scratch_bytes() { return kNoAllocScratchBytes; }

bool gemm_noalloc(const Nvfp4DeviceOperands& op, cudaStream_t s, std::string* err) {
  const int cc = device_cc_major(err);
  if (cc == 0) return false;
  if (cc != 10) {
    set_err(err, "the b200 backend needs an sm_100 device (found sm_" + std::to_string(cc) + "x)");
    return false;
  }
  if (op.out_dtype == OutDType::NVFP4) {
    set_err(err, "NVFP4 output is not supported by the no-alloc GEMM (FP32 or BF16 only)");
    return false;
  }
  if (op.mode != GemmMode::Dense) {
    set_err(err, "the no-alloc GEMM supports dense mode only");
    return false;
  }
  if (op.sf_layout != SfLayout::Canonical) {
    set_err(err, "the no-alloc GEMM takes canonical [rows][K/16] scales "
                 "(tcgen05-layout scales need no scratch: use nvfp4_b200_gemm)");
    return false;
  }
  if (!op.a_packed || !op.b_packed || !op.a_scales || !op.b_scales) {
    set_err(err, "null operand pointer");
    return false;
  }
  void* out = op.d ? op.d : static_cast<void*>(op.c);
  if (!out) {
    set_err(err, "null output pointer");
    return false;
  }
  if (op.M <= 0 || op.N <= 0 || op.K <= 0 || op.K % 32 != 0) {
    set_err(err, "M, N, K must be positive and K a multiple of 32");
    return false;
  }
  if ((reinterpret_cast<uintptr_t>(op.a_packed) | reinterpret_cast<uintptr_t>(op.b_packed)) & 15) {
    set_err(err, "packed operands must be 16-byte aligned");
    return false;
  }
  const size_t na = round256(sf_tcgen05_bytes(op.M, op.K));
  const size_t nb = round256(sf_tcgen05_bytes(op.N, op.K));
  if (na + nb > kNoAllocScratchBytes) {
    set_err(err, "problem too large for the no-alloc GEMM: its reordered scales need " +
                     std::to_string(na + nb) + " bytes, the fixed scratch holds " +
                     std::to_string(kNoAllocScratchBytes) +
                     " ((M+N)*K/16 must stay under about 16 Mi)");
    return false;
  }
  uint8_t* scratch = scratch_for_current_device(err);
  if (!scratch) return false;
  if (!sf_to_tcgen05_pair(op.a_scales, op.M, op.b_scales, op.N, op.K, scratch, scratch + na, s, err))
    return false;
  return gemm_dense_tc(op, scratch, scratch + na, out, s, err);
}

}  // namespace nvfp4b200
