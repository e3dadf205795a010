// roofs.cu - the two measured roofs of the roofline: HBM bandwidth and tcgen05 FP4 throughput.
//
// HBM roof: replaces the reference's STREAM triad (src/bandwidth.cu:6-52) with three
// vectorised (128-bit) grid-stride kernels over caller buffers much larger than L2: copy
// (read + write), read-only (a reduction whose single result per CTA is written), and the
// reference's triad c = a + s*b. GB/s counts every byte read or written once.
//
// Compute roof: replaces the reference's register-resident mma.sync ladder
// (src/peak.cu:23-156, which cannot run on sm_100a) with a memory-free tcgen05 rung: each CTA
// stages one zeroed A/B tile and its scales once, then one elected thread issues `iters`
// tcgen05.mma kind::mxf4nvf4 block_scale (M=128, N=n, K=64) back to back into one TMEM
// accumulator and waits for their completion through tcgen05.commit. Throughput does not
// depend on the data.
#include <cuda_runtime.h>

#include <algorithm>
#include <string>

#include "internal.h"
#include "ptx.cuh"

namespace nvfp4b200 {
namespace {

__global__ void copy_kernel(const uint4* __restrict__ src, uint4* __restrict__ dst, size_t n) {
  for (size_t i = blockIdx.x * size_t(blockDim.x) + threadIdx.x; i < n;
       i += size_t(gridDim.x) * blockDim.x)
    dst[i] = src[i];
}

__global__ void read_kernel(const uint4* __restrict__ src, size_t n, uint32_t* __restrict__ sink) {
  uint32_t acc = 0;
  for (size_t i = blockIdx.x * size_t(blockDim.x) + threadIdx.x; i < n;
       i += size_t(gridDim.x) * blockDim.x) {
    const uint4 v = src[i];
    acc ^= v.x ^ v.y ^ v.z ^ v.w;
  }
  acc = __reduce_xor_sync(0xffffffffu, acc);
  if ((threadIdx.x & 31) == 0 && acc == 0x9E3779B9u) sink[blockIdx.x] = acc;  // keeps the loads live
}

__global__ void triad_kernel(const float4* __restrict__ a, const float4* __restrict__ b,
                             float4* __restrict__ c, float s, size_t n) {
  for (size_t i = blockIdx.x * size_t(blockDim.x) + threadIdx.x; i < n;
       i += size_t(gridDim.x) * blockDim.x) {
    const float4 x = a[i], y = b[i];
    c[i] = make_float4(x.x + s * y.x, x.y + s * y.y, x.z + s * y.z, x.w + s * y.w);
  }
}

constexpr int kPeakThreads = 128;

template <int N>
__global__ void __launch_bounds__(kPeakThreads, 1) peak_kernel(int iters, uint32_t* err_word) {
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) &
                                             ~uintptr_t(1023));
  constexpr int kA = 128 * 128, kB = N * 128, kSf = 4096;
  uint64_t* bar = reinterpret_cast<uint64_t*>(smem + kA + kB + kSf);
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(bar + 1);
  for (int i = threadIdx.x; i < (kA + kB + kSf) / 16; i += blockDim.x)
    reinterpret_cast<uint4*>(smem)[i] = make_uint4(0, 0, 0, 0);
  // Unit scales (UE4M3 1.0 = 0x38) so the accumulator stays finite.
  for (int i = threadIdx.x; i < kSf; i += blockDim.x) smem[kA + kB + i] = 0x38;
  if (threadIdx.x == 0) {
    mbar_init(smem_u32(bar), 1);
    fence_mbar_init();
  }
  asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
  if (threadIdx.x < 32) {
    tmem_alloc(smem_u32(tmem_slot), 512);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tbase = *tmem_slot;
  if (threadIdx.x == 0) {
    const uint32_t a_s = smem_u32(smem), b_s = smem_u32(smem + kA), sf_s = smem_u32(smem + kA + kB);
    const uint32_t sfa_t = tbase + 448, sfb_t = tbase + 456;
    tc_cp_32x128b_x4(sfa_t, make_sdesc(sf_s, 16, 128, 0));
    tc_cp_32x128b_x4(sfb_t, make_sdesc(sf_s + 512, 16, 128, 0));
    tc_cp_32x128b_x4(sfb_t + 4, make_sdesc(sf_s + 1024, 16, 128, 0));
    const uint32_t idesc = make_idesc_mxf4nvf4(128, N);
    const uint64_t ad = make_sdesc(a_s, 16, 1024, 2), bd = make_sdesc(b_s, 16, 1024, 2);
    for (int i = 0; i < iters; ++i) tc_mma_mxf4nvf4(tbase, ad, bd, idesc, sfa_t, sfb_t, i > 0);
    tc_commit(smem_u32(bar));
    volatile int never = 0;
    mbar_wait(smem_u32(bar), 0, &never, err_word, kErrWaitDrain);
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  if (threadIdx.x < 32) tmem_dealloc(tbase, 512);
}

// SM-pair rung: clusters of two CTAs; the leader issues M=256 x N x K=64 MMAs with
// cta_group::2 (each SM computes 128 x N), both CTAs allocate TMEM and hold scale copies.
template <int N>
__global__ void __launch_bounds__(kPeakThreads, 1) peak_pair_kernel(int iters, uint32_t* err_word) {
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) &
                                             ~uintptr_t(1023));
  constexpr int kA = 128 * 128, kB = (N / 2) * 128, kSf = 4096;
  uint64_t* bar = reinterpret_cast<uint64_t*>(smem + kA + kB + kSf);
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(bar + 1);
  for (int i = threadIdx.x; i < (kA + kB) / 16; i += blockDim.x)
    reinterpret_cast<uint4*>(smem)[i] = make_uint4(0, 0, 0, 0);
  if (threadIdx.x == 0) {
    mbar_init(smem_u32(bar), 1);
    fence_mbar_init();
  }
  if (threadIdx.x < 32) {
    tmem_alloc_pair(smem_u32(tmem_slot), 512);
    tmem_relinquish_pair();
  }
  tc_fence_before();
  __syncthreads();
  cluster_sync();
  tc_fence_after();
  const uint32_t tbase = *tmem_slot;
  // Unit scales (0x38) into TMEM rows of both CTAs by their own threads.
  if (threadIdx.x < 128) {
    const int q = threadIdx.x >> 5;
    const uint32_t lb = tbase + (static_cast<uint32_t>(q * 32) << 16) + 448;
    uint32_t v[16];
    for (int i = 0; i < 16; ++i) v[i] = 0x38383838u;
    tmem_st_32x32b_x16(lb, v);
    tc_wait_st();
  }
  tc_fence_before();
  __syncthreads();
  cluster_sync();
  tc_fence_after();
  if (threadIdx.x == 0 && cluster_ctarank() == 0) {
    const uint32_t a_s = smem_u32(smem), b_s = smem_u32(smem + kA);
    const uint32_t idesc = make_idesc_mxf4nvf4(256, N);
    const uint64_t ad = make_sdesc(a_s, 16, 1024, 2), bd = make_sdesc(b_s, 16, 1024, 2);
    for (int i = 0; i < iters; ++i)
      tc_mma_mxf4nvf4_pair(tbase, ad, bd, idesc, tbase + 448, tbase + 452, i > 0);
    tc_commit_pair(smem_u32(bar));
    volatile int never = 0;
    mbar_wait(smem_u32(bar), 0, &never, err_word, kErrWaitDrain);
  }
  tc_fence_before();
  __syncthreads();
  cluster_sync();
  tc_fence_after();
  if (threadIdx.x < 32) tmem_dealloc_pair(tbase, 512);
}

}  // namespace

bool peak_ladder_pair(int n, int clusters, int iters, int reps, double* tflops, cudaStream_t s,
                      std::string* err) {
  if (n != 256 || clusters < 1 || iters < 1 || reps < 1 || !tflops) {
    set_err(err, "peak (pair): n must be 256, clusters/iters/reps >= 1");
    return false;
  }
  uint32_t* ew = device_error_word(err);
  if (!ew) return false;
  const int smem = 1024 + 128 * 128 + 128 * 128 + 4096 + 64;
  cudaError_t e = cudaFuncSetAttribute(peak_pair_kernel<256>,
                                       cudaFuncAttributeMaxDynamicSharedMemorySize, smem);
  if (e != cudaSuccess) {
    set_err(err, std::string("peak pair attr: ") + cudaGetErrorString(e));
    return false;
  }
  cudaLaunchConfig_t cfg = {};
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeClusterDimension;
  attr[0].val.clusterDim.x = 2;
  attr[0].val.clusterDim.y = 1;
  attr[0].val.clusterDim.z = 1;
  cfg.gridDim = dim3(2 * clusters, 1, 1);
  cfg.blockDim = dim3(kPeakThreads, 1, 1);
  cfg.dynamicSmemBytes = smem;
  cfg.stream = s;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  auto launch = [&]() { return cudaLaunchKernelEx(&cfg, peak_pair_kernel<256>, iters, ew); };
  if ((e = launch()) != cudaSuccess) {
    set_err(err, std::string("peak pair launch: ") + cudaGetErrorString(e));
    return false;
  }
  cudaEvent_t a, b;
  cudaEventCreate(&a);
  cudaEventCreate(&b);
  float best = 1e30f;
  for (int r = 0; r < reps; ++r) {
    cudaEventRecord(a, s);
    launch();
    cudaEventRecord(b, s);
    cudaEventSynchronize(b);
    float ms = 0;
    cudaEventElapsedTime(&ms, a, b);
    best = std::min(best, ms);
  }
  cudaEventDestroy(a);
  cudaEventDestroy(b);
  e = cudaGetLastError();
  if (e != cudaSuccess) {
    set_err(err, std::string("peak pair: ") + cudaGetErrorString(e));
    return false;
  }
  *tflops = 2.0 * 256.0 * n * 64.0 * static_cast<double>(clusters) * iters / (best * 1e-3) / 1e12;
  return true;
}

bool measure_bandwidth(int kind, const void* src, void* dst, const void* src2, size_t bytes,
                       int iters, double* gbs, cudaStream_t s, std::string* err) {
  if (!src || !gbs || (kind != 1 && !dst) || (kind == 2 && !src2) || kind < 0 || kind > 2) {
    set_err(err, "measure_bandwidth: bad arguments");
    return false;
  }
  if (((reinterpret_cast<uintptr_t>(src) | reinterpret_cast<uintptr_t>(dst) |
        reinterpret_cast<uintptr_t>(src2)) & 15) || bytes < 16 || iters < 1) {
    set_err(err, "measure_bandwidth: buffers must be 16-byte aligned, bytes >= 16, iters >= 1");
    return false;
  }
  int dev = 0, sms = 148;
  cudaGetDevice(&dev);
  cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
  const size_t n = bytes / 16;
  const int block = 512, grid = sms * 4;
  uint32_t* sink = static_cast<uint32_t*>(dst);
  auto launch = [&]() {
    if (kind == 0)
      copy_kernel<<<grid, block, 0, s>>>(static_cast<const uint4*>(src), static_cast<uint4*>(dst), n);
    else if (kind == 1)
      read_kernel<<<grid, block, 0, s>>>(static_cast<const uint4*>(src), n, sink);
    else
      triad_kernel<<<grid, block, 0, s>>>(static_cast<const float4*>(src),
                                          static_cast<const float4*>(src2),
                                          static_cast<float4*>(dst), 1.5f, n);
  };
  if (kind == 1 && !dst) {
    set_err(err, "read-only probe needs dst as a sink of >= 4*SMs*4 bytes");
    return false;
  }
  for (int i = 0; i < 3; ++i) launch();
  cudaEvent_t a, b;
  cudaEventCreate(&a);
  cudaEventCreate(&b);
  float best = 1e30f;
  for (int i = 0; i < iters; ++i) {
    cudaEventRecord(a, s);
    launch();
    cudaEventRecord(b, s);
    cudaEventSynchronize(b);
    float ms = 0;
    cudaEventElapsedTime(&ms, a, b);
    best = std::min(best, ms);
  }
  cudaEventDestroy(a);
  cudaEventDestroy(b);
  cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) {
    set_err(err, std::string("measure_bandwidth: ") + cudaGetErrorString(e));
    return false;
  }
  const double moved = static_cast<double>(n) * 16.0 * (kind == 0 ? 2.0 : kind == 1 ? 1.0 : 3.0);
  *gbs = moved / (best * 1e-3) / 1e9;
  return true;
}

bool peak_ladder(int n, int ctas, int iters, int reps, double* tflops, cudaStream_t s,
                 std::string* err) {
  if ((n != 128 && n != 256) || ctas < 1 || iters < 1 || reps < 1 || !tflops) {
    set_err(err, "peak: n must be 128 or 256, ctas/iters/reps >= 1");
    return false;
  }
  uint32_t* ew = device_error_word(err);
  if (!ew) return false;
  const int smem = 1024 + 128 * 128 + n * 128 + 4096 + 64;
  cudaError_t e;
  if (n == 256)
    e = cudaFuncSetAttribute(peak_kernel<256>, cudaFuncAttributeMaxDynamicSharedMemorySize, smem);
  else
    e = cudaFuncSetAttribute(peak_kernel<128>, cudaFuncAttributeMaxDynamicSharedMemorySize, smem);
  if (e != cudaSuccess) {
    set_err(err, std::string("peak attr: ") + cudaGetErrorString(e));
    return false;
  }
  auto launch = [&]() {
    if (n == 256) peak_kernel<256><<<ctas, kPeakThreads, smem, s>>>(iters, ew);
    else peak_kernel<128><<<ctas, kPeakThreads, smem, s>>>(iters, ew);
  };
  launch();
  cudaEvent_t a, b;
  cudaEventCreate(&a);
  cudaEventCreate(&b);
  float best = 1e30f;
  for (int r = 0; r < reps; ++r) {
    cudaEventRecord(a, s);
    launch();
    cudaEventRecord(b, s);
    cudaEventSynchronize(b);
    float ms = 0;
    cudaEventElapsedTime(&ms, a, b);
    best = std::min(best, ms);
  }
  cudaEventDestroy(a);
  cudaEventDestroy(b);
  e = cudaGetLastError();
  if (e != cudaSuccess) {
    set_err(err, std::string("peak: ") + cudaGetErrorString(e));
    return false;
  }
  const double flops = 2.0 * 128.0 * n * 64.0 * static_cast<double>(ctas) * iters;
  *tflops = flops / (best * 1e-3) / 1e12;
  return true;
}

}  // namespace nvfp4b200
