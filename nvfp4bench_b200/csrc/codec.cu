// codec.cu - NVFP4 codecs on the GPU, byte-identical to the reference's host codecs.
//
// Restated from src/nvfp4.cu (reference project):
//   e2m1_quantize  :18-29  nearest of {0,.5,1,1.5,2,3,4,6}, ties to the smaller magnitude
//   e4m3_decode    :34-45  UE4M3, bias 7, subnormals; code 0x7F decodes to 480
//   e4m3_encode    :47-59  nearest code in 0..127, ties to the lower code, x clamped to 448
//   quantize       :62-97  per-16 amax -> scale (amax/6)/g -> code -> x / (dec(code)*g)
//   dequantize     :99-112
//   make_random    :115-129 splitmix64 -> uniform [-1, 1)
// Every float operation is the same IEEE single operation as in the host code (explicit
// __fdiv_rn / __fmul_rn, no contraction), so bytes match exactly. The per-element division
// x / dec feeds only the E2M1 midpoint comparisons, which are made exactly on |x| against
// per-block thresholds instead (e2m1_quantize_scaled). The linear 128-way scale
// search becomes a rounding of the float's bits to the UE4M3 grid with ties to the lower code
// (codec_dev.cuh), which picks the same code: decoded values strictly increase with the code,
// so the nearest code is one of the two grid points around x, and the errors the reference
// compares are exact float differences there.
#include <cuda_runtime.h>

#include <string>

#include "codec_dev.cuh"
#include "internal.h"

namespace nvfp4b200 {
namespace {

__global__ void fill_uniform_kernel(float* __restrict__ out, size_t n, uint64_t x0) {
  for (size_t i = blockIdx.x * size_t(blockDim.x) + threadIdx.x; i < n;
       i += size_t(gridDim.x) * blockDim.x) {
    const uint64_t z = splitmix_mix(x0 + static_cast<uint64_t>(i + 1) * kGolden);
    out[i] = __fsub_rn(__fmul_rn(__fdiv_rn(static_cast<float>(z >> 40), 16777216.0f), 2.0f), 1.0f);
  }
}

__global__ void fill_normal_kernel(float* __restrict__ out, size_t n, uint64_t x0) {
  const size_t pairs = (n + 1) / 2;
  for (size_t p = blockIdx.x * size_t(blockDim.x) + threadIdx.x; p < pairs;
       p += size_t(gridDim.x) * blockDim.x) {
    const uint64_t z1 = splitmix_mix(x0 + static_cast<uint64_t>(2 * p + 1) * kGolden);
    const uint64_t z2 = splitmix_mix(x0 + static_cast<uint64_t>(2 * p + 2) * kGolden);
    const float u1 = (static_cast<float>(z1 >> 40) + 1.0f) * (1.0f / 16777216.0f);  // (0, 1]
    const float u2 = static_cast<float>(z2 >> 40) * (1.0f / 16777216.0f);           // [0, 1)
    const float r = sqrtf(-2.0f * logf(u1));
    float sn, cs;
    sincospif(2.0f * u2, &sn, &cs);
    out[2 * p] = r * cs;
    if (2 * p + 1 < n) out[2 * p + 1] = r * sn;
  }
}

// One thread per BLK-element block (src/nvfp4.cu:66-95 with BLK = 16; BLK = 32 is the scale
// block of the sparse tensor-core MMA). ka = tcgen05 atoms per 128-row block along K.
template <int BLK>
__global__ void quantize_kernel(const float* __restrict__ src, int rows, int cols, float g,
                                uint8_t* __restrict__ packed, uint8_t* __restrict__ scales,
                                uint8_t* __restrict__ scales_tc, int ka) {
  // Launched with programmatic stream serialization: read the source only once the previous
  // kernel has completed, and let the next kernel (typically the GEMM reading these bytes,
  // which waits for this grid the same way) start its set-up now.
  asm volatile("griddepcontrol.wait;" ::: "memory");
  asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
  const int nb = cols / BLK;
  const size_t nblocks = static_cast<size_t>(rows) * nb;
  const size_t stride = size_t(gridDim.x) * blockDim.x;
  // (row, block) of the grid-stride index, advanced by the stride's quotient and remainder
  // instead of a 64-bit division per block.
  const size_t blk0 = blockIdx.x * size_t(blockDim.x) + threadIdx.x;
  int r = static_cast<int>(blk0 / nb), b = static_cast<int>(blk0 % nb);
  const int dr = static_cast<int>(stride / nb), db = static_cast<int>(stride % nb);
  for (size_t blk = blk0; blk < nblocks; blk += stride) {
    const float4* x4 = reinterpret_cast<const float4*>(src + static_cast<size_t>(r) * cols + b * BLK);
    float x[BLK];
#pragma unroll
    for (int v = 0; v < BLK / 4; ++v) {
      const float4 t = x4[v];
      x[4 * v] = t.x; x[4 * v + 1] = t.y; x[4 * v + 2] = t.z; x[4 * v + 3] = t.w;
    }
    float amax = 0.0f;
#pragma unroll
    for (int j = 0; j < BLK; ++j) {
      const float a = fabsf(x[j]);
      if (amax < a) amax = a;  // std::max(amax, a): NaN never replaces amax
    }
    const float scale = (amax > 0.0f) ? __fdiv_rn(__fdiv_rn(amax, 6.0f), g) : 1.0f;
    const uint8_t sc = e4m3_encode_dev(scale);
    float dec = __fmul_rn(e4m3_decode_dev(sc), g);
    if (dec <= 0.0f) dec = 1.0f;
    const E2m1Thresholds th = e2m1_thresholds(dec);
    const bool fast = amax < th.big;
    uint32_t w[BLK / 8];
#pragma unroll
    for (int q = 0; q < BLK / 8; ++q) w[q] = e2m1_pack8(x + 8 * q, dec, th, fast);
    uint8_t* dst = packed + (static_cast<size_t>(r) * cols + b * BLK) / 2;
    if (BLK == 16) *reinterpret_cast<uint2*>(dst) = make_uint2(w[0], w[1]);
    else *reinterpret_cast<uint4*>(dst) = make_uint4(w[0], w[1], w[BLK / 8 > 2 ? 2 : 0], w[BLK / 8 > 3 ? 3 : 0]);
    if (scales) scales[blk] = sc;
    if (scales_tc) {
      const size_t atom = static_cast<size_t>(r / 128) * ka + b / 4;
      scales_tc[atom * 512 + (r % 32) * 16 + ((r / 32) % 4) * 4 + (b % 4)] = sc;
    }
    r += dr;
    b += db;
    if (b >= nb) {
      b -= nb;
      ++r;
    }
  }
}

// src/nvfp4.cu:99-112, one thread per 16-element half-block of a BLK-element scale block.
template <int BLK>
__global__ void dequantize_kernel(const uint8_t* __restrict__ packed, const uint8_t* __restrict__ scales,
                                  int rows, int cols, float g, float* __restrict__ out) {
  const int nh = cols / 16;
  const size_t nhalves = static_cast<size_t>(rows) * nh;
  for (size_t h = blockIdx.x * size_t(blockDim.x) + threadIdx.x; h < nhalves;
       h += size_t(gridDim.x) * blockDim.x) {
    const size_t r = h / nh, c0 = (h % nh) * 16;
    const float s = __fmul_rn(e4m3_decode_dev(scales[r * (cols / BLK) + c0 / BLK]), g);
    const size_t e0 = r * static_cast<size_t>(cols) + c0;
    const uint2 w = *reinterpret_cast<const uint2*>(packed + e0 / 2);
    float4* o = reinterpret_cast<float4*>(out + e0);
#pragma unroll
    for (int v = 0; v < 4; ++v) {
      const uint32_t word = v < 2 ? w.x : w.y;
      const int sh = (v & 1) * 16;
      o[v] = make_float4(__fmul_rn(e2m1_decode_dev((word >> sh) & 0xF), s),
                         __fmul_rn(e2m1_decode_dev((word >> (sh + 4)) & 0xF), s),
                         __fmul_rn(e2m1_decode_dev((word >> (sh + 8)) & 0xF), s),
                         __fmul_rn(e2m1_decode_dev((word >> (sh + 12)) & 0xF), s));
    }
  }
}

// ---- pair-wise 2:4 sparsity (the pattern of the tcgen05 .sp kind::mxf4nvf4 MMA) ----------
// Each group of 8 consecutive K elements of an A row is 4 element pairs, 2 of them kept.
// Group i (row-major over rows x K/8) keeps combination splitmix64(seed + (i+1)*golden) % 6 of
// {01, 02, 03, 12, 13, 23}; its metadata nibble is first | second << 2, two groups per byte.
__constant__ uint8_t kSpLo[6] = {0, 0, 0, 1, 1, 2};
__constant__ uint8_t kSpHi[6] = {1, 2, 3, 2, 3, 3};

__global__ void sparse_meta_kernel(uint8_t* __restrict__ meta, size_t nbytes, uint64_t seed) {
  for (size_t j = blockIdx.x * size_t(blockDim.x) + threadIdx.x; j < nbytes;
       j += size_t(gridDim.x) * blockDim.x) {
    uint32_t b = 0;
#pragma unroll
    for (int h = 0; h < 2; ++h) {
      const uint64_t i = 2 * j + h;
      const unsigned p = static_cast<unsigned>(splitmix_mix(seed + (i + 1) * kGolden) % 6);
      b |= static_cast<uint32_t>(kSpLo[p] | (kSpHi[p] << 2)) << (4 * h);
    }
    meta[j] = static_cast<uint8_t>(b);
  }
}

// Zero the two dropped pairs of every group of an fp32 [rows][K] matrix, in place.
__global__ void sparse_prune_kernel(float* __restrict__ a, const uint8_t* __restrict__ meta, size_t ngroups) {
  for (size_t i = blockIdx.x * size_t(blockDim.x) + threadIdx.x; i < ngroups;
       i += size_t(gridDim.x) * blockDim.x) {
    const uint32_t nib = (meta[i / 2] >> (4 * (i & 1))) & 0xF;
    float4* g4 = reinterpret_cast<float4*>(a + i * 8);
    float4 lo = g4[0], hi = g4[1];
    const uint32_t keep = (1u << (nib & 3)) | (1u << ((nib >> 2) & 3));
    if (!(keep & 1u)) { lo.x = 0.0f; lo.y = 0.0f; }
    if (!(keep & 2u)) { lo.z = 0.0f; lo.w = 0.0f; }
    if (!(keep & 4u)) { hi.x = 0.0f; hi.y = 0.0f; }
    if (!(keep & 8u)) { hi.z = 0.0f; hi.w = 0.0f; }
    g4[0] = lo;
    g4[1] = hi;
  }
}

// packed [rows][K/2] -> values [rows][K/4]: one pair is one byte; a metadata byte (2 groups)
// turns 8 packed bytes into 4 value bytes.
__global__ void sparse_compress_kernel(const uint8_t* __restrict__ packed, const uint8_t* __restrict__ meta,
                                       uint8_t* __restrict__ values, size_t nbytes) {
  for (size_t j = blockIdx.x * size_t(blockDim.x) + threadIdx.x; j < nbytes;
       j += size_t(gridDim.x) * blockDim.x) {
    const uint32_t m = meta[j];
    const uint2 w = *reinterpret_cast<const uint2*>(packed + 8 * j);
    auto byte_of = [](uint32_t word, uint32_t k) { return (word >> (8 * k)) & 0xFFu; };
    const uint32_t v = byte_of(w.x, m & 3) | (byte_of(w.x, (m >> 2) & 3) << 8) |
                       (byte_of(w.y, (m >> 4) & 3) << 16) | (byte_of(w.y, (m >> 6) & 3) << 24);
    *reinterpret_cast<uint32_t*>(values + 4 * j) = v;
  }
}

// One block per (128-row block, 16 scale atoms): the 128 x 64 canonical scale bytes are read
// row by row (coalesced) into shared memory, then written out as 16 whole 512-byte atoms
// (coalesced). Rows past `rows` and scales past `ns` are written as zero.
constexpr int kSfTileAtoms = 16;
__device__ __forceinline__ void sf_tile(const uint8_t* __restrict__ scales, int rows, int ns, int ka,
                                        uint32_t* __restrict__ out, int rb, int a0) {
  __shared__ uint32_t tile[128][kSfTileAtoms + 1];  // [row][atom]: the row's 4 scales of the atom
  const int s0 = a0 * 4;
  if ((ns & 3) == 0 && (reinterpret_cast<uintptr_t>(scales) & 3) == 0) {
    // Whole rows of 4-scale words (K a multiple of 64): one word per (row, atom), all of a
    // thread's loads issued before any is stored, so the block waits on memory once.
    const uint32_t* s32 = reinterpret_cast<const uint32_t*>(scales);
    constexpr int kWords = 128 * kSfTileAtoms;
    constexpr int kPer = kWords / 256;
    uint32_t v[kPer];
#pragma unroll
    for (int i = 0; i < kPer; ++i) {
      const int idx = threadIdx.x + i * 256;
      const int r = idx / kSfTileAtoms, a = idx % kSfTileAtoms;
      const int row = rb * 128 + r;
      v[i] = (row < rows && a0 + a < ka) ? s32[static_cast<size_t>(row) * ka + a0 + a] : 0u;
    }
#pragma unroll
    for (int i = 0; i < kPer; ++i) {
      const int idx = threadIdx.x + i * 256;
      tile[idx / kSfTileAtoms][idx % kSfTileAtoms] = v[i];
    }
  } else {
  uint8_t* tb = reinterpret_cast<uint8_t*>(&tile[0][0]);
  for (int idx = threadIdx.x; idx < 128 * kSfTileAtoms * 4; idx += blockDim.x) {
    const int r = idx / (kSfTileAtoms * 4), c = idx % (kSfTileAtoms * 4);
    const int row = rb * 128 + r, sc = s0 + c;
    uint8_t v = 0;
    if (row < rows && sc < ns) v = scales[static_cast<size_t>(row) * ns + sc];
    tb[(r * (kSfTileAtoms + 1) + c / 4) * 4 + (c & 3)] = v;
  }
  }
  __syncthreads();
  for (int w = threadIdx.x; w < kSfTileAtoms * 128; w += blockDim.x) {
    const int a = w >> 7, wi = w & 127;
    if (a0 + a >= ka) break;
    const int r = (wi & 3) * 32 + (wi >> 2);
    out[(static_cast<size_t>(rb) * ka + a0 + a) * 128 + wi] = tile[r][a];
  }
}

// One block per (128-row block, 16 scale atoms) of one operand (blockIdx.z: 0 = first,
// 1 = second, so both GEMM operands are reordered in one launch): the 128 x 64 canonical
// scale bytes are read row by row (coalesced) into shared memory, then written out as 16 whole
// 512-byte atoms (coalesced). Rows past `rows` and scales past `ns` are written as zero.
__global__ void __launch_bounds__(256) sf_to_tcgen05_kernel(const uint8_t* __restrict__ s0_, int rows0,
                                                             uint32_t* __restrict__ out0,
                                                             const uint8_t* __restrict__ s1_, int rows1,
                                                             uint32_t* __restrict__ out1, int ns, int ka) {
  // The GEMM that reads the reordered scales is launched with programmatic stream
  // serialization and waits for this grid to complete before reading them; letting it launch
  // now overlaps its set-up with this kernel.
  asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
  const bool second = blockIdx.z == 1;
  const int rows = second ? rows1 : rows0;
  if (static_cast<int>(blockIdx.y) * 128 >= rows) return;
  sf_tile(second ? s1_ : s0_, rows, ns, ka, second ? out1 : out0, blockIdx.y,
          blockIdx.x * kSfTileAtoms);
}

int grid_for(size_t work, int block) {
  size_t g = (work + block - 1) / block;
  if (g > 148 * 32) g = 148 * 32;
  if (g < 1) g = 1;
  return static_cast<int>(g);
}

bool check_launch(const char* what, std::string* err) {
  cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) {
    set_err(err, std::string(what) + ": " + cudaGetErrorString(e));
    return false;
  }
  return true;
}

}  // namespace

bool fill_uniform(float* out, size_t n, uint64_t seed, cudaStream_t s, std::string* err) {
  if (!out) { set_err(err, "null output"); return false; }
  if (n == 0) return true;
  const uint64_t x0 = seed ? seed : kGolden;  // src/nvfp4.cu:118
  fill_uniform_kernel<<<grid_for(n, 256), 256, 0, s>>>(out, n, x0);
  return check_launch("fill_uniform", err);
}

bool fill_normal(float* out, size_t n, uint64_t seed, cudaStream_t s, std::string* err) {
  if (!out) { set_err(err, "null output"); return false; }
  if (n == 0) return true;
  const uint64_t x0 = seed ? seed : kGolden;
  fill_normal_kernel<<<grid_for((n + 1) / 2, 256), 256, 0, s>>>(out, n, x0);
  return check_launch("fill_normal", err);
}

bool quantize_block(const float* src, int rows, int cols, float global_scale, int block,
                    uint8_t* packed, uint8_t* scales, uint8_t* scales_tc, cudaStream_t s,
                    std::string* err) {
  if (!src || !packed) { set_err(err, "null pointer"); return false; }
  if (block != 16 && block != 32) { set_err(err, "quantize block must be 16 or 32"); return false; }
  if (rows < 0 || cols < 0 || cols % block != 0) {
    set_err(err, "quantize needs rows >= 0 and cols a multiple of the block (16 or 32)");
    return false;
  }
  if ((reinterpret_cast<uintptr_t>(src) & 15) || (reinterpret_cast<uintptr_t>(packed) & (block == 16 ? 7 : 15))) {
    set_err(err, "quantize needs a 16-byte aligned source and an 8-byte (16-byte for block 32) aligned packed output");
    return false;
  }
  const size_t nblocks = static_cast<size_t>(rows) * (cols / block);
  if (nblocks == 0) return true;
  // Block 32: atoms of 128 rows x 4 scales cover 128 K, the same atom layout over cols / 2.
  const int vcols = block == 16 ? cols : cols / 2;
  // The tcgen05 layout pads rows to 128 and scales to 4 per row: zero it only when there is
  // padding that the kernel does not write.
  if (scales_tc && (rows % 128 != 0 || (vcols / 16) % 4 != 0)) {
    if (cudaMemsetAsync(scales_tc, 0, sf_tcgen05_bytes(rows, vcols), s) != cudaSuccess) {
      set_err(err, "cudaMemsetAsync of the tcgen05 scale buffer failed");
      return false;
    }
  }
  const int ka = (vcols + 63) / 64;
  cudaLaunchConfig_t cfg = {};
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.gridDim = dim3(grid_for(nblocks, 256), 1, 1);
  cfg.blockDim = dim3(256, 1, 1);
  cfg.stream = s;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  cudaError_t e = block == 16
      ? cudaLaunchKernelEx(&cfg, quantize_kernel<16>, src, rows, cols, global_scale, packed, scales,
                           scales_tc, ka)
      : cudaLaunchKernelEx(&cfg, quantize_kernel<32>, src, rows, cols, global_scale, packed, scales,
                           scales_tc, ka);
  if (e != cudaSuccess) {
    set_err(err, std::string("quantize launch: ") + cudaGetErrorString(e));
    return false;
  }
  return check_launch("quantize", err);
}

bool quantize(const float* src, int rows, int cols, float global_scale, uint8_t* packed,
              uint8_t* scales, uint8_t* scales_tc, cudaStream_t s, std::string* err) {
  return quantize_block(src, rows, cols, global_scale, 16, packed, scales, scales_tc, s, err);
}

bool dequantize_block(const uint8_t* packed, const uint8_t* scales, int rows, int cols,
                      float global_scale, int block, float* out, cudaStream_t s, std::string* err) {
  if (!packed || !scales || !out) { set_err(err, "null pointer"); return false; }
  if (block != 16 && block != 32) { set_err(err, "dequantize block must be 16 or 32"); return false; }
  if (rows < 0 || cols < 0 || cols % block != 0) {
    set_err(err, "dequantize needs cols a multiple of the block (16 or 32)");
    return false;
  }
  if ((reinterpret_cast<uintptr_t>(out) & 15) || (reinterpret_cast<uintptr_t>(packed) & 7)) {
    set_err(err, "dequantize needs a 16-byte aligned output and an 8-byte aligned packed input");
    return false;
  }
  const size_t nhalves = static_cast<size_t>(rows) * (cols / 16);
  if (nhalves == 0) return true;
  if (block == 16)
    dequantize_kernel<16><<<grid_for(nhalves, 256), 256, 0, s>>>(packed, scales, rows, cols,
                                                                global_scale, out);
  else
    dequantize_kernel<32><<<grid_for(nhalves, 256), 256, 0, s>>>(packed, scales, rows, cols,
                                                                global_scale, out);
  return check_launch("dequantize", err);
}

bool dequantize(const uint8_t* packed, const uint8_t* scales, int rows, int cols,
                float global_scale, float* out, cudaStream_t s, std::string* err) {
  return dequantize_block(packed, scales, rows, cols, global_scale, 16, out, s, err);
}

bool sparse_meta(int rows, int K, uint64_t seed, uint8_t* meta, cudaStream_t s, std::string* err) {
  if (!meta) { set_err(err, "null pointer"); return false; }
  if (rows < 0 || K < 0 || K % 16 != 0) {
    set_err(err, "sparse metadata needs K a multiple of 16");
    return false;
  }
  const size_t nbytes = static_cast<size_t>(rows) * (K / 16);
  if (nbytes == 0) return true;
  sparse_meta_kernel<<<grid_for(nbytes, 256), 256, 0, s>>>(meta, nbytes, seed);
  return check_launch("sparse_meta", err);
}

bool sparse_prune(float* a, int rows, int K, const uint8_t* meta, cudaStream_t s, std::string* err) {
  if (!a || !meta) { set_err(err, "null pointer"); return false; }
  if (rows < 0 || K < 0 || K % 16 != 0 || (reinterpret_cast<uintptr_t>(a) & 15)) {
    set_err(err, "sparse prune needs K a multiple of 16 and a 16-byte aligned matrix");
    return false;
  }
  const size_t ngroups = static_cast<size_t>(rows) * (K / 8);
  if (ngroups == 0) return true;
  sparse_prune_kernel<<<grid_for(ngroups, 256), 256, 0, s>>>(a, meta, ngroups);
  return check_launch("sparse_prune", err);
}

bool sparse_compress(const uint8_t* packed, int rows, int K, const uint8_t* meta, uint8_t* values,
                     cudaStream_t s, std::string* err) {
  if (!packed || !meta || !values) { set_err(err, "null pointer"); return false; }
  if (rows < 0 || K < 0 || K % 16 != 0 || (reinterpret_cast<uintptr_t>(packed) & 7) ||
      (reinterpret_cast<uintptr_t>(values) & 3)) {
    set_err(err, "sparse compress needs K a multiple of 16, packed 8-byte and values 4-byte aligned");
    return false;
  }
  const size_t nbytes = static_cast<size_t>(rows) * (K / 16);
  if (nbytes == 0) return true;
  sparse_compress_kernel<<<grid_for(nbytes, 256), 256, 0, s>>>(packed, meta, values, nbytes);
  return check_launch("sparse_compress", err);
}

bool sf_to_tcgen05(const uint8_t* scales, int rows, int K, uint8_t* out, cudaStream_t s,
                   std::string* err) {
  return sf_to_tcgen05_pair(scales, rows, nullptr, 0, K, out, nullptr, s, err);
}

bool sf_to_tcgen05_pair(const uint8_t* a, int rows_a, const uint8_t* b, int rows_b, int K,
                        uint8_t* out_a, uint8_t* out_b, cudaStream_t s, std::string* err) {
  if (!a || !out_a || (b && !out_b)) { set_err(err, "null pointer"); return false; }
  if (rows_a <= 0 || (b && rows_b <= 0) || K <= 0 || K % 16 != 0) {
    set_err(err, "sf_to_tcgen05 needs rows > 0 and K a positive multiple of 16");
    return false;
  }
  if ((reinterpret_cast<uintptr_t>(out_a) | reinterpret_cast<uintptr_t>(out_b)) & 3) {
    set_err(err, "tcgen05 scale output must be 4-byte aligned");
    return false;
  }
  const int ka = (K + 63) / 64;
  const int rmax = b && rows_b > rows_a ? rows_b : rows_a;
  const dim3 grid((ka + kSfTileAtoms - 1) / kSfTileAtoms, (rmax + 127) / 128, b ? 2 : 1);
  sf_to_tcgen05_kernel<<<grid, 256, 0, s>>>(a, rows_a, reinterpret_cast<uint32_t*>(out_a), b,
                                            b ? rows_b : 0, reinterpret_cast<uint32_t*>(out_b),
                                            K / 16, ka);
  return check_launch("sf_to_tcgen05", err);
}

}  // namespace nvfp4b200

// ---- GPU mirror of the reference oracle (src/reference.cu:9-17) for the C++ harness's
// --validate: C[m][n] = sum_k A[m][k] * B[n][k] in FP32, k ascending, one thread per output.
namespace nvfp4b200 {
namespace {
__global__ void naive_gemm_nt_kernel(const float* __restrict__ A, const float* __restrict__ B,
                                     float* __restrict__ C, int M, int N, int K) {
  const int n = blockIdx.x * blockDim.x + threadIdx.x, m = blockIdx.y * blockDim.y + threadIdx.y;
  if (m >= M || n >= N) return;
  float acc = 0.0f;
  for (int k = 0; k < K; ++k) acc = __fadd_rn(acc, __fmul_rn(A[static_cast<size_t>(m) * K + k],
                                                            B[static_cast<size_t>(n) * K + k]));
  C[static_cast<size_t>(m) * N + n] = acc;
}
}  // namespace

bool naive_gemm_nt(const float* A, const float* B, int M, int N, int K, float* C, cudaStream_t s,
                   std::string* err) {
  dim3 block(16, 16), grid((N + 15) / 16, (M + 15) / 16);
  naive_gemm_nt_kernel<<<grid, block, 0, s>>>(A, B, C, M, N, K);
  return check_launch("naive_gemm_nt", err);
}
}  // namespace nvfp4b200
