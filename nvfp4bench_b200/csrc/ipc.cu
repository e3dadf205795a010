// ipc.cu - CUDA IPC export/import of device buffers (C ABI, include/nvfp4_b200.h), so that the
// ranks of a column-sharded GEMM can write their output tiles straight into each other's
// output buffers (the fused all-gather). No reference counterpart: the reference runs one GPU.
#include <cuda.h>
#include <cuda_runtime.h>

#include <cstdint>
#include <cstring>
#include <map>
#include <mutex>
#include <string>

#include "nvfp4_b200.h"

namespace {

static_assert(sizeof(cudaIpcMemHandle_t) == NVFP4_B200_IPC_HANDLE_BYTES, "IPC handle size");

int put_err(int code, const std::string& msg, char* err, size_t errlen) {
  if (err && errlen) {
    const size_t n = msg.size() < errlen - 1 ? msg.size() : errlen - 1;
    std::memcpy(err, msg.data(), n);
    err[n] = '\0';
  }
  return code;
}

using AddressRangeFn = CUresult (*)(CUdeviceptr*, size_t*, CUdeviceptr);

AddressRangeFn address_range_fn() {
  static AddressRangeFn fn = nullptr;
  static std::once_flag once;
  std::call_once(once, [] {
    void* ptr = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPointByVersion("cuMemGetAddressRange", &ptr, 12000, cudaEnableDefault,
                                         &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<AddressRangeFn>(ptr);
  });
  return fn;
}

// One mapping per imported allocation (CUDA maps an allocation at most once per process),
// keyed by its handle bytes and shared by every open of a pointer inside it.
struct Mapping {
  char* base = nullptr;
  int refs = 0;
};
std::mutex g_mu;
std::map<std::string, Mapping> g_by_handle;
struct Opened {
  std::string key;  // handle of the allocation
  int refs = 0;     // opens that returned this address
};
std::map<uintptr_t, Opened> g_opened;

}  // namespace

extern "C" {

int nvfp4_b200_ipc_handle(const void* ptr, void* handle, size_t* offset, char* err, size_t errlen) {
  if (!ptr || !handle || !offset) return put_err(NVFP4_B200_EINVAL, "null argument", err, errlen);
  AddressRangeFn range = address_range_fn();
  if (!range) return put_err(NVFP4_B200_ECUDA, "cuMemGetAddressRange unavailable", err, errlen);
  CUdeviceptr base = 0;
  size_t size = 0;
  if (range(&base, &size, reinterpret_cast<CUdeviceptr>(ptr)) != CUDA_SUCCESS)
    return put_err(NVFP4_B200_EINVAL, "pointer is not device memory of this process", err, errlen);
  cudaIpcMemHandle_t h;
  cudaError_t e = cudaIpcGetMemHandle(&h, reinterpret_cast<void*>(base));
  if (e != cudaSuccess)
    return put_err(NVFP4_B200_ECUDA, std::string("cudaIpcGetMemHandle: ") + cudaGetErrorString(e),
                   err, errlen);
  std::memcpy(handle, &h, sizeof(h));
  *offset = static_cast<size_t>(reinterpret_cast<CUdeviceptr>(ptr) - base);
  if (err && errlen) err[0] = '\0';
  return NVFP4_B200_OK;
}

int nvfp4_b200_ipc_open(const void* handle, size_t offset, void** ptr, char* err, size_t errlen) {
  if (!handle || !ptr) return put_err(NVFP4_B200_EINVAL, "null argument", err, errlen);
  const std::string key(static_cast<const char*>(handle), NVFP4_B200_IPC_HANDLE_BYTES);
  std::lock_guard<std::mutex> lk(g_mu);
  Mapping& m = g_by_handle[key];
  if (m.refs == 0) {
    cudaIpcMemHandle_t h;
    std::memcpy(&h, handle, sizeof(h));
    void* base = nullptr;
    cudaError_t e = cudaIpcOpenMemHandle(&base, h, cudaIpcMemLazyEnablePeerAccess);
    if (e != cudaSuccess) {
      g_by_handle.erase(key);
      return put_err(NVFP4_B200_ECUDA,
                     std::string("cudaIpcOpenMemHandle: ") + cudaGetErrorString(e), err, errlen);
    }
    m.base = static_cast<char*>(base);
  }
  ++m.refs;
  *ptr = m.base + offset;
  Opened& o = g_opened[reinterpret_cast<uintptr_t>(*ptr)];
  o.key = key;
  ++o.refs;
  if (err && errlen) err[0] = '\0';
  return NVFP4_B200_OK;
}

int nvfp4_b200_ipc_close(void* ptr, char* err, size_t errlen) {
  std::lock_guard<std::mutex> lk(g_mu);
  auto it = g_opened.find(reinterpret_cast<uintptr_t>(ptr));
  if (it == g_opened.end())
    return put_err(NVFP4_B200_EINVAL, "pointer was not returned by nvfp4_b200_ipc_open", err, errlen);
  const std::string key = it->second.key;
  if (--it->second.refs == 0) g_opened.erase(it);
  auto m = g_by_handle.find(key);
  if (m != g_by_handle.end() && --m->second.refs == 0) {
    cudaError_t e = cudaIpcCloseMemHandle(m->second.base);
    g_by_handle.erase(m);
    if (e != cudaSuccess)
      return put_err(NVFP4_B200_ECUDA,
                     std::string("cudaIpcCloseMemHandle: ") + cudaGetErrorString(e), err, errlen);
  }
  if (err && errlen) err[0] = '\0';
  return NVFP4_B200_OK;
}

}  // extern "C"
