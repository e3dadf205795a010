// roofs.cu - the two measured roofs of the roofline: HBM bandwidth and tcgen05 FP4 throughput.
//
// HBM roof: replaces the reference's STREAM triad (src/bandwidth.cu:6-52) with three
// vectorised (128-bit) grid-stride kernels over caller buffers much larger than L2: copy
// (read + write), read-only (a reduction whose single result per CTA is written), and the
// reference's triad c = a + s*b. GB/s counts every byte read or written once.
//
// Compute roof: replaces the reference's register-resident mma.sync ladder
// (src/peak.cu:23-156, which cannot run on sm_100a) with a memory-free tcgen05 rung: each CTA
// stages one A/B tile and its scales once, then one elected thread issues `iters`
// tcgen05.mma kind::mxf4nvf4 block_scale (M=128, N=n, K=64) back to back into one TMEM
// accumulator and waits for their completion through tcgen05.commit. The tile is zero or, with
// a non-zero seed, pseudo-random E2M1 bytes: the issue rate does not depend on the data, but
// the power drawn does, and under the 1 kW cap the SM clock (which the rung reports, from
// clock64 against globaltimer on CTA 0) falls with it. The random-data rung, timed as the mean
// of back-to-back launches, is the sustained FP4 roof for a GEMM on real operands.
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

__device__ unsigned long long g_peak_clk[2];  // CTA 0 of the last rung: SM cycles, ns

// Fill `bytes` (a multiple of 16) of shared memory with zeros or seeded pseudo-random bytes.
__device__ __forceinline__ void fill_tile(uint8_t* dst, int bytes, uint32_t seed) {
  for (int i = threadIdx.x; i < bytes / 4; i += blockDim.x) {
    uint32_t x = 0;
    if (seed) {
      x = (static_cast<uint32_t>(i) + blockIdx.x * 0x01000193u) * 0x9E3779B1u ^ seed;
      x ^= x >> 16;
      x *= 0x85EBCA6Bu;
      x ^= x >> 13;
      x *= 0xC2B2AE35u;
      x ^= x >> 16;
    }
    reinterpret_cast<uint32_t*>(dst)[i] = x;
  }
}

__device__ __forceinline__ void record_clock(long long c0, uint64_t n0) {
  if (blockIdx.x == 0) {
    g_peak_clk[0] = static_cast<unsigned long long>(clock64() - c0);
    g_peak_clk[1] = globaltimer_ns() - n0;
  }
}

__device__ __forceinline__ void peak_mma_sp(uint32_t d, uint64_t a, uint64_t b, uint32_t meta, uint32_t idesc,
                                            uint32_t sfa, uint32_t sfb, uint32_t acc) {
  asm volatile(
      "{\n\t.reg .pred p;\n\tsetp.ne.b32 p, %7, 0;\n\t"
      "tcgen05.mma.sp.cta_group::1.kind::mxf4nvf4.block_scale.scale_vec::4X "
      "[%0], %1, %2, [%3], %4, [%5], [%6], p;\n\t}" ::"r"(d),
      "l"(a), "l"(b), "r"(meta), "r"(idesc), "r"(sfa), "r"(sfb), "r"(acc)
      : "memory");
}

// SP: the sparse rung (tcgen05.mma.sp, 128 logical K per MMA: A holds the kept half).
template <int N, bool SP = false>
__global__ void __launch_bounds__(kPeakThreads, 1) peak_kernel(int iters, uint32_t seed, uint32_t* err_word) {
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) &
                                             ~uintptr_t(1023));
  constexpr int kA = 128 * 128, kB = N * 128, kSf = 4096;
  uint64_t* bar = reinterpret_cast<uint64_t*>(smem + kA + kB + kSf);
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(bar + 1);
  fill_tile(smem, kA + kB, seed);
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
  if (SP) {
    // Valid pair metadata (pairs 0 and 1 of every group) in the rows' own lanes.
    const uint32_t lb = tbase + (static_cast<uint32_t>((threadIdx.x >> 5) * 32) << 16) + 464;
    uint32_t v[4] = {0x44444444u, 0x44444444u, 0x44444444u, 0x44444444u};
    tmem_st_32x32b_x4(lb, v[0], v[1], v[2], v[3]);
    tc_wait_st();
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
  }
  if (threadIdx.x == 0) {
    const uint32_t a_s = smem_u32(smem), b_s = smem_u32(smem + kA), sf_s = smem_u32(smem + kA + kB);
    const uint32_t sfa_t = tbase + 448, sfb_t = tbase + 456;
    tc_cp_32x128b_x4(sfa_t, make_sdesc(sf_s, 16, 128, 0));
    tc_cp_32x128b_x4(sfb_t, make_sdesc(sf_s + 512, 16, 128, 0));
    tc_cp_32x128b_x4(sfb_t + 4, make_sdesc(sf_s + 1024, 16, 128, 0));
    const uint32_t idesc = make_idesc_mxf4nvf4(128, N);
    const uint64_t ad = make_sdesc(a_s, 16, 1024, 2), bd = make_sdesc(b_s, 16, 1024, 2);
    const long long c0 = clock64();
    const uint64_t n0 = globaltimer_ns();
    if (SP)
      for (int i = 0; i < iters; ++i) peak_mma_sp(tbase, ad, bd, tbase + 464, idesc | (1u << 2), sfa_t, sfb_t, i > 0);
    else
      for (int i = 0; i < iters; ++i) tc_mma_mxf4nvf4(tbase, ad, bd, idesc, sfa_t, sfb_t, i > 0);
    tc_commit(smem_u32(bar));
    volatile int never = 0;
    mbar_wait(smem_u32(bar), 0, &never, err_word, kErrWaitDrain);
    record_clock(c0, n0);
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  if (threadIdx.x < 32) tmem_dealloc(tbase, 512);
}

// SM-pair rung: clusters of two CTAs; the leader issues M=256 x N x K=64 MMAs with
// cta_group::2 (each SM computes 128 x N), both CTAs allocate TMEM and hold scale copies.
template <int N>
__global__ void __launch_bounds__(kPeakThreads, 1) peak_pair_kernel(int iters, uint32_t seed, uint32_t* err_word) {
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) &
                                             ~uintptr_t(1023));
  constexpr int kA = 128 * 128, kB = (N / 2) * 128, kSf = 4096;
  uint64_t* bar = reinterpret_cast<uint64_t*>(smem + kA + kB + kSf);
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(bar + 1);
  fill_tile(smem, kA + kB, seed);
  asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
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
    const long long c0 = clock64();
    const uint64_t n0 = globaltimer_ns();
    for (int i = 0; i < iters; ++i)
      tc_mma_mxf4nvf4_pair(tbase, ad, bd, idesc, tbase + 448, tbase + 452, i > 0);
    tc_commit_pair(smem_u32(bar));
    volatile int never = 0;
    mbar_wait(smem_u32(bar), 0, &never, err_word, kErrWaitDrain);
    record_clock(c0, n0);
  }
  tc_fence_before();
  __syncthreads();
  cluster_sync();
  tc_fence_after();
  if (threadIdx.x < 32) tmem_dealloc_pair(tbase, 512);
}

}  // namespace

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

bool peak_ladder_ex(const PeakOptions& o, double* tflops, double* sm_mhz, cudaStream_t s,
                    std::string* err) {
  const bool pair = o.cta_group == 2;
  if ((o.cta_group != 1 && !pair) || (pair ? o.n != 256 : (o.n != 128 && o.n != 256)) ||
      o.units < 1 || o.iters < 1 || o.reps < 1 || !tflops || (o.sparse && pair)) {
    set_err(err, "peak: cta_group 1 (n 128 or 256, dense or sparse) or 2 (n 256, dense); "
                 "units, iters, reps >= 1");
    return false;
  }
  uint32_t* ew = device_error_word(err);
  if (!ew) return false;
  const int kb = pair ? o.n / 2 : o.n;
  const int smem = 1024 + 128 * 128 + kb * 128 + 4096 + 64;
  void (*kern)(int, uint32_t, uint32_t*) =
      pair ? peak_pair_kernel<256>
           : o.sparse ? (o.n == 256 ? peak_kernel<256, true> : peak_kernel<128, true>)
                      : (o.n == 256 ? peak_kernel<256> : peak_kernel<128>);
  cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, smem);
  if (e != cudaSuccess) {
    set_err(err, std::string("peak attr: ") + cudaGetErrorString(e));
    return false;
  }
  cudaLaunchConfig_t cfg = {};
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeClusterDimension;
  attr[0].val.clusterDim.x = 2;
  attr[0].val.clusterDim.y = 1;
  attr[0].val.clusterDim.z = 1;
  cfg.gridDim = dim3(pair ? 2 * o.units : o.units, 1, 1);
  cfg.blockDim = dim3(kPeakThreads, 1, 1);
  cfg.dynamicSmemBytes = smem;
  cfg.stream = s;
  cfg.attrs = pair ? attr : nullptr;
  cfg.numAttrs = pair ? 1 : 0;
  const uint32_t seed = o.seed;
  auto launch = [&]() { return cudaLaunchKernelEx(&cfg, kern, o.iters, seed, ew); };
  if ((e = launch()) != cudaSuccess) {
    set_err(err, std::string("peak launch: ") + cudaGetErrorString(e));
    return false;
  }
  cudaEvent_t a, b;
  cudaEventCreate(&a);
  cudaEventCreate(&b);
  float ms_used = 1e30f;
  if (o.sustained) {
    // Back-to-back launches between one pair of events: the mean, under the power cap.
    cudaEventRecord(a, s);
    for (int r = 0; r < o.reps; ++r) launch();
    cudaEventRecord(b, s);
    cudaEventSynchronize(b);
    float ms = 0;
    cudaEventElapsedTime(&ms, a, b);
    ms_used = ms / o.reps;
  } else {
    for (int r = 0; r < o.reps; ++r) {
      cudaEventRecord(a, s);
      launch();
      cudaEventRecord(b, s);
      cudaEventSynchronize(b);
      float ms = 0;
      cudaEventElapsedTime(&ms, a, b);
      ms_used = std::min(ms_used, ms);
    }
  }
  cudaEventDestroy(a);
  cudaEventDestroy(b);
  e = cudaGetLastError();
  if (e != cudaSuccess) {
    set_err(err, std::string("peak: ") + cudaGetErrorString(e));
    return false;
  }
  const double m = pair ? 256.0 : 128.0;
  const double k = o.sparse ? 128.0 : 64.0;   // logical K per MMA
  *tflops = 2.0 * m * o.n * k * static_cast<double>(o.units) * o.iters / (ms_used * 1e-3) / 1e12;
  if (sm_mhz) {
    unsigned long long clk[2] = {0, 0};
    cudaMemcpyFromSymbol(clk, g_peak_clk, sizeof(clk));
    *sm_mhz = clk[1] ? 1e3 * static_cast<double>(clk[0]) / static_cast<double>(clk[1]) : 0.0;
  }
  return true;
}

bool peak_ladder(int n, int ctas, int iters, int reps, double* tflops, cudaStream_t s,
                 std::string* err) {
  return peak_ladder_ex(PeakOptions{n, 1, ctas, iters, reps, 0u, 0, 0}, tflops, nullptr, s, err);
}

bool peak_ladder_pair(int n, int clusters, int iters, int reps, double* tflops, cudaStream_t s,
                      std::string* err) {
  return peak_ladder_ex(PeakOptions{n, 2, clusters, iters, reps, 0u, 0, 0}, tflops, nullptr, s, err);
}

}  // namespace nvfp4b200
