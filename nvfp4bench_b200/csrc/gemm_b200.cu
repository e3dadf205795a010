// gemm_b200.cu - the B200 backend: NVFP4 block-scaled GEMM on 5th-generation tensor cores.
//
// D[M x N] = alpha * A[M x K] * B[N x K]^T with E2M1 operands and UE4M3 scales per 16
// K-elements, FP32 accumulation in Tensor Memory, alpha = a_global * b_global applied in the
// epilogue. Drop-in for the reference's backend slot: launch_gemm_b200 has the signature of
// launch_gemm_custom (src/gemm.h:27-29) and honours its ownership and error rules
// (src/gemm.h:25-26: return false + message, never throw, never exit, async on the stream).
//
// Kernel design (one persistent CTA per SM, 448 threads):
//   warp 0      TMA producer: per K-stage, two tiled TMA loads (A 128 x 256 FP4, B BN x 256
//               FP4, both 128-byte-swizzled K-major) completing on one mbarrier ("full").
//               Four 48 KB stages (BN = 256) or six 32 KB stages (BN = 128). No multicast.
//   warp 1      MMA issuer (one lane): per K-stage, four tcgen05.mma kind::mxf4nvf4
//               block_scale (M=128, N=BN, K=64) back to back. One tcgen05.commit per stage
//               frees the smem stage and its TMEM scale slot ("empty") and, per tile,
//               publishes the accumulator ("acc_full").
//   warps 2..5  epilogue: tcgen05.ld 32 lanes x 32 columns, scale by alpha, convert to
//               FP32/BF16, write the 32 x 32 chunk into a swizzled, double-buffered shared
//               tile and store it with one TMA tensor store (clipped at the matrix edges).
//               Warp w reads TMEM lane quadrant w % 4. Outputs whose row pitch is not a
//               multiple of 16 bytes fall back to per-thread global stores.
//   warps 6..13 scale writers, two per TMEM quadrant taking even and odd stages in turn:
//               per K-stage each loads its lanes' 16 bytes of the stage's scale atoms from
//               global memory (L2) into registers and writes them with tcgen05.st into a
//               ring of two scale slots in TMEM (one batched store per stage: a cross-warp
//               mbarrier round trip costs ~390 cycles, more than the 128-cycle MMA a
//               per-K-block handshake would feed). Each warp writes its own 32-lane quadrant.
//               SFB rows map to accumulator columns, which every quadrant computes, so SFB is
//               stored whole in all four quadrants (the layout tcgen05.cp .warpx4 produces);
//               SFA rows map to TMEM lanes, and the MMA rows of quadrant q read only column q
//               of each 4-column SFA group, so each writer stores just that column (a quarter
//               of the bytes; verified bit-exact by the integer known-answer test).
//               The kernel ran 16% faster with no scale stores at all (an isolated MMA stream
//               is not slowed by concurrent TMEM stores; the interaction inside the kernel is
//               not isolated yet), and fewer bytes measured faster. tcgen05.cp
//               would do the copy on the tensor pipe, in series with the MMAs (4 MMAs of a
//               stage take 512 cycles, 980 with the stage's 12 copies). Scales take no shared
//               memory, which leaves room for a fourth A/B stage: more bytes in flight for the
//               L2-to-shared-memory stream.
// Two accumulator buffers let the epilogue of tile i overlap the MMAs of tile i+1. With
// BN = 256 the two 256-column buffers and the 96 scale columns do not fit the 512 TMEM
// columns side by side, so buffer 1 starts at column 160: the epilogue loads the 3 chunks
// that hold the 96 shared columns first, releases them ("acc_early") as soon as they are in
// registers, and drains the rest afterwards.
//
// The same kernel with SP = true is the pair-wise 2:4 sparse GEMM (tcgen05.mma.sp; see its
// section below), and any of the kernels can write C as NVFP4 (store_chunk_nvfp4).
//
// Every mbarrier wait is bounded (ptx.cuh); a timeout sets the device error word, all roles
// leave their loops, in-flight copies and MMAs are drained with bounded waits, TMEM is freed
// and the kernel returns.
#include <cuda.h>
#include <cuda_bf16.h>
#include <cuda_runtime.h>

#include <cstdio>
#include <cstring>
#include <mutex>
#include <string>
#include <vector>

#include "gemm.h"
#include "internal.h"
#include "codec_dev.cuh"
#include "ptx.cuh"

namespace nvfp4b200 {

__device__ uint32_t g_device_error = 0;

namespace {

constexpr int kBM = 128;          // rows of A per tile (= TMEM lanes)
constexpr int kBKBytes = 128;     // one K-stage = 256 FP4 = 128 bytes per row (one swizzle atom)
constexpr int kKBlocksPerStage = 4;  // MMA K = 64 -> 4 MMAs per stage
constexpr int kNumThreads = 448;  // 14 warps
constexpr int kWriterGroups = 2;  // scale writers: two warps per TMEM quadrant, even/odd stages
constexpr int kTmemCols = 512;
constexpr int kSfSlotCols = 48;   // per stage: SFA at +4*kb (16 columns), SFB at +16 + 8*kb
constexpr int kSfbOff = 16;
#ifndef NVFP4_SF_SLOTS
#define NVFP4_SF_SLOTS 2
#endif
#ifndef NVFP4_PAIR_SF_SLOTS
#define NVFP4_PAIR_SF_SLOTS NVFP4_SF_SLOTS
#endif

// SP: the sparse variant (tcgen05.mma.sp, pair-wise 2:4 A): a stage is 256 logical K, A
// compressed to 64 bytes per row (one 64-byte-swizzled TMA box), two sparse MMAs of N = BN.
template <int BN, bool SP = false>
struct Cfg {
  static constexpr int kABytes = kBM * (SP ? 64 : kBKBytes);     // 16 KB (8 KB compressed)
  static constexpr int kBBytes = BN * kBKBytes;                  // 16 / 32 KB
  static constexpr int kStageBytes = kABytes + kBBytes;          // scales bypass smem
  static constexpr int kStages = (BN == 256) ? 4 : 6;
  static constexpr int kCBufBytes = 32 * 32 * 4;                // per epilogue warp: 2 BF16 / 1 FP32 chunk
  static constexpr int kCBytes = 4 * kCBufBytes;                // 4 epilogue warps
  // The stage's B scale atoms ((BN / 128) row blocks x the stage's atoms along K x 512 bytes),
  // brought in once per CTA by bulk copy; every scale-writer quadrant reads them from shared
  // memory.
  // (Sparse: the scale atoms along K are per 128 logical K, two per stage.)
  static constexpr int kSfbAtomsPerStage = SP ? 2 : kKBlocksPerStage;
  static constexpr int kSfbStageBytes = ((BN + 127) / 128) * kSfbAtomsPerStage * 512;
  static constexpr int kSfbBytes = kStages * kSfbStageBytes;
  static constexpr int kBarBytes = 512;
  static constexpr int kSmemBytes = 1024 + kStages * kStageBytes + kCBytes + kSfbBytes + kBarBytes;
  // TMEM: a ring of scale slots at the top (slot it % kSfSlots, freed with the smem stage
  // that used it last), two accumulator buffers below; which 32-column chunks the buffers share.
  static constexpr int kSfSlots = NVFP4_SF_SLOTS;
  static_assert(kSfSlots <= kStages, "a writer's slot wait must also order its full[] arrival");
  static constexpr int kSfCol = kTmemCols - kSfSlots * kSfSlotCols;  // 368
  static constexpr int kAccBase1 = (BN == 256) ? kSfCol - 256 : BN;  // 112 for BN = 256
  static constexpr int kChunks = BN / 32;
  static constexpr bool kOverlap = (BN == 256);
  // Buffer 0's last and buffer 1's first kOverlapChunks chunks hold the shared columns.
  static constexpr int kOverlapChunks = (256 - kAccBase1 + 31) / 32;
  static constexpr int kSfbAtoms = (BN + 127) / 128;
  static constexpr int kSfbColsPerKb = kSfbAtoms * 4;
  static_assert(kSmemBytes <= 232448, "shared memory budget");
  static_assert(kAccBase1 + BN <= kSfCol && kAccBase1 >= 0, "TMEM budget");
  static_assert(!kOverlap || (kOverlapChunks >= 3 && kOverlapChunks <= 6), "overlap chunks");
};

struct GemmParams {
  const uint8_t* sfa;   // tcgen05 scale layout
  const uint8_t* sfb;
  void* out;
  int M, N, K;
  int ldc;
  float alpha;
  int out_bf16;
  int tma_store;        // 1: epilogue stores through the C tensor map
  int tiles_m, tiles_n, num_tiles;
  int group_m;
  int ka;               // scale atoms along K = ceil(K/64) (sparse: ceil(K/128))
  const uint8_t* meta;  // sparse: pair metadata [M][K/16]
  int out_nvfp4;        // 1: `out` is packed NVFP4 [M][N/2] with scales out_sf
  uint8_t* out_sf;
  float out_g;          // its global scale
  int out_sf_tc;        // out_sf in the tcgen05 layout (else canonical [M][N/16])
  int out_ka;           // tcgen05 scale atoms per 128-row block of the output = ceil(N/64)
  int num_kt;           // K-stages = ceil(K/256)
  int sfb_rowblocks;    // ceil(N/128)
  int sfa_rowblocks;    // ceil(M/128)
  uint32_t* err_word;
  // Further destinations of every output tile (TMA-store path only): tensor maps in global
  // memory, one per destination, with the same coordinates as the C map.
  const CUtensorMap* peer_maps;
  int n_peers;
};

__device__ __forceinline__ void tile_coords(const GemmParams& p, int t, int& tm, int& tn) {
  const int per_group = p.group_m * p.tiles_n;
  const int g = t / per_group;
  const int first_m = g * p.group_m;
  int gsize = p.tiles_m - first_m;
  if (gsize > p.group_m) gsize = p.group_m;
  const int local = t - g * per_group;
  tm = first_m + local % gsize;
  tn = local / gsize;
}

// Bounded wait that ignores the abort flag (used to drain in-flight work after an abort).
__device__ __forceinline__ bool mbar_wait_drain(uint32_t bar, uint32_t parity, uint32_t* err) {
  volatile int never = 0;
  return mbar_wait(bar, parity, &never, err, kErrWaitDrain);
}

__device__ __forceinline__ uint32_t pack_bf16x2(float lo, float hi) {
  __nv_bfloat162 v = __floats2bfloat162_rn(lo, hi);
  return *reinterpret_cast<uint32_t*>(&v);
}

// Scale one 32-column chunk of a row by alpha and store it (vector stores when the chunk is
// whole and the row is aligned, element stores at the ragged edges).
__device__ __forceinline__ void store_chunk(const GemmParams& p, const uint32_t (&r)[32], int row,
                                            int col0) {
  if (row >= p.M || col0 >= p.N) return;
  const bool full_chunk = col0 + 32 <= p.N;
  if (p.out_bf16) {
    __nv_bfloat16* out =
        reinterpret_cast<__nv_bfloat16*>(p.out) + static_cast<size_t>(row) * p.ldc + col0;
    if (full_chunk && (p.ldc % 8) == 0) {
      uint4* o = reinterpret_cast<uint4*>(out);
#pragma unroll
      for (int v = 0; v < 4; ++v) {
        uint4 w;
        w.x = pack_bf16x2(__uint_as_float(r[8 * v + 0]) * p.alpha, __uint_as_float(r[8 * v + 1]) * p.alpha);
        w.y = pack_bf16x2(__uint_as_float(r[8 * v + 2]) * p.alpha, __uint_as_float(r[8 * v + 3]) * p.alpha);
        w.z = pack_bf16x2(__uint_as_float(r[8 * v + 4]) * p.alpha, __uint_as_float(r[8 * v + 5]) * p.alpha);
        w.w = pack_bf16x2(__uint_as_float(r[8 * v + 6]) * p.alpha, __uint_as_float(r[8 * v + 7]) * p.alpha);
        o[v] = w;
      }
    } else {
#pragma unroll
      for (int jj = 0; jj < 32; ++jj)
        if (col0 + jj < p.N) out[jj] = __float2bfloat16_rn(__uint_as_float(r[jj]) * p.alpha);
    }
  } else {
    float* out = reinterpret_cast<float*>(p.out) + static_cast<size_t>(row) * p.ldc + col0;
    if (full_chunk && (p.ldc % 4) == 0) {
      float4* o = reinterpret_cast<float4*>(out);
#pragma unroll
      for (int v = 0; v < 8; ++v)
        o[v] = make_float4(__uint_as_float(r[4 * v + 0]) * p.alpha, __uint_as_float(r[4 * v + 1]) * p.alpha,
                           __uint_as_float(r[4 * v + 2]) * p.alpha, __uint_as_float(r[4 * v + 3]) * p.alpha);
    } else {
#pragma unroll
      for (int jj = 0; jj < 32; ++jj)
        if (col0 + jj < p.N) out[jj] = __uint_as_float(r[jj]) * p.alpha;
    }
  }
}

// NVFP4 output: the chunk's two 16-column blocks of row `row` quantised exactly as
// quantize_to_nvfp4 (src/nvfp4.cu:62-97, shared device code): 16 packed bytes and 2 scale
// bytes. N % 32 == 0, so a chunk is wholly inside or outside the matrix.
__device__ __forceinline__ void store_chunk_nvfp4(const GemmParams& p, const uint32_t (&r)[32], int row,
                                                  int col0) {
  if (row >= p.M || col0 >= p.N) return;
  float x0[16], x1[16];
#pragma unroll
  for (int j = 0; j < 16; ++j) {
    x0[j] = __fmul_rn(__uint_as_float(r[j]), p.alpha);
    x1[j] = __fmul_rn(__uint_as_float(r[16 + j]), p.alpha);
  }
  uint32_t a0, a1, b0, b1;
  const uint32_t s0 = quantize16_dev(x0, p.out_g, a0, a1);
  const uint32_t s1 = quantize16_dev(x1, p.out_g, b0, b1);
  uint8_t* out = reinterpret_cast<uint8_t*>(p.out);
  *reinterpret_cast<uint4*>(out + (static_cast<size_t>(row) * p.N + col0) / 2) = make_uint4(a0, a1, b0, b1);
  const int s = col0 / 16;
  size_t off;
  if (p.out_sf_tc)
    off = (static_cast<size_t>(row / 128) * p.out_ka + s / 4) * 512 + (row % 32) * 16 +
          ((row / 32) % 4) * 4 + (s % 4);
  else
    off = static_cast<size_t>(row) * (p.N / 16) + s;
  *reinterpret_cast<uint16_t*>(p.out_sf + off) = static_cast<uint16_t>(s0 | (s1 << 8));
}

// Per-warp epilogue state for the TMA-store path: two 4 KB staging buffers used in turn.
struct EpiStage {
  uint8_t* buf;        // this warp's two buffers
  uint32_t count;      // chunks stored so far
  const void* tmap_c;
  int row0;            // first row of this warp's 32-row slab
};

// Scale one 32 x 32 chunk (lane = row) by alpha, write it to a staging buffer in the TMA
// swizzled layout (64-byte swizzle for BF16 rows of 64 bytes, 128-byte for FP32 rows of 128
// bytes; either way one st.shared.v4 per 16 bytes without bank conflicts) and store it (and,
// with kPeers, to every peer destination).
template <bool kPeers = true>
__device__ __forceinline__ void stage_chunk(const GemmParams& p, EpiStage& e, const uint32_t (&r)[32],
                                            int col0) {
  const int lane = threadIdx.x & 31;
  // A warp's 4 KB staging area holds two BF16 chunks (2 KB each, used in turn) or one FP32 chunk.
  // With peer destinations a BF16 warp also stages 64-column pairs there (stage_pair), so every
  // chunk then waits for all earlier stores to have read the whole area.
  const bool dbl = p.out_bf16 != 0 && !(kPeers && p.n_peers > 0);
  uint8_t* b = e.buf + (dbl ? (e.count & 1) * 2048 : 0);
  if (lane == 0) {  // the store that last used this buffer has read it
    if (dbl) bulk_wait_group_read<1>();
    else bulk_wait_group_read<0>();
  }
  __syncwarp();
  if (p.out_bf16) {
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      uint4 w;
      w.x = pack_bf16x2(__uint_as_float(r[8 * j + 0]) * p.alpha, __uint_as_float(r[8 * j + 1]) * p.alpha);
      w.y = pack_bf16x2(__uint_as_float(r[8 * j + 2]) * p.alpha, __uint_as_float(r[8 * j + 3]) * p.alpha);
      w.z = pack_bf16x2(__uint_as_float(r[8 * j + 4]) * p.alpha, __uint_as_float(r[8 * j + 5]) * p.alpha);
      w.w = pack_bf16x2(__uint_as_float(r[8 * j + 6]) * p.alpha, __uint_as_float(r[8 * j + 7]) * p.alpha);
      *reinterpret_cast<uint4*>(b + lane * 64 + ((j ^ ((lane >> 1) & 3)) << 4)) = w;
    }
  } else {
#pragma unroll
    for (int j = 0; j < 8; ++j)
      *reinterpret_cast<float4*>(b + lane * 128 + ((j ^ (lane & 7)) << 4)) =
          make_float4(__uint_as_float(r[4 * j + 0]) * p.alpha, __uint_as_float(r[4 * j + 1]) * p.alpha,
                      __uint_as_float(r[4 * j + 2]) * p.alpha, __uint_as_float(r[4 * j + 3]) * p.alpha);
  }
  fence_proxy_async_smem();
  __syncwarp();
  if (lane == 0) {
    tma_store_2d(e.tmap_c, smem_u32(b), col0, e.row0);
    // The fused all-gather: the same staged chunk to every peer destination (stores over
    // NVLink by the TMA unit; one commit group covers them all).
    // Compiled out of the kernels launched without peers: the loop alone cost the C2 GEMM 2%.
    if constexpr (kPeers)
      for (int r = 0; r < p.n_peers; ++r) tma_store_2d(p.peer_maps + r, smem_u32(b), col0, e.row0);
    bulk_commit_group();
  }
  ++e.count;
}

// BF16 output with peer destinations: two adjacent 32-column chunks staged as one 32 x 64 tile
// (128-byte rows, 128-byte swizzle) and stored with one 64-column box to this GPU's C and to
// every peer. A 64-byte row per box used about half of an NVLink's bandwidth; 128-byte rows
// carry FP32 output at about 0.8 of it. The wide maps follow the narrow peer maps in
// p.peer_maps: [n narrow peers][n wide peers][wide local C].
__device__ __forceinline__ void stage_pair(const GemmParams& p, EpiStage& e, const uint32_t (&r0)[32],
                                           const uint32_t (&r1)[32], int col0) {
  const int lane = threadIdx.x & 31;
  uint8_t* b = e.buf;
  if (lane == 0) bulk_wait_group_read<0>();
  __syncwarp();
#pragma unroll
  for (int j = 0; j < 8; ++j) {
    const uint32_t* r = j < 4 ? r0 : r1;
    const int o = 8 * (j & 3);
    uint4 w;
    w.x = pack_bf16x2(__uint_as_float(r[o + 0]) * p.alpha, __uint_as_float(r[o + 1]) * p.alpha);
    w.y = pack_bf16x2(__uint_as_float(r[o + 2]) * p.alpha, __uint_as_float(r[o + 3]) * p.alpha);
    w.z = pack_bf16x2(__uint_as_float(r[o + 4]) * p.alpha, __uint_as_float(r[o + 5]) * p.alpha);
    w.w = pack_bf16x2(__uint_as_float(r[o + 6]) * p.alpha, __uint_as_float(r[o + 7]) * p.alpha);
    *reinterpret_cast<uint4*>(b + lane * 128 + ((j ^ (lane & 7)) << 4)) = w;
  }
  fence_proxy_async_smem();
  __syncwarp();
  if (lane == 0) {
    const int n = p.n_peers;
    tma_store_2d(p.peer_maps + 2 * n, smem_u32(b), col0, e.row0);
    for (int i = 0; i < n; ++i) tma_store_2d(p.peer_maps + n + i, smem_u32(b), col0, e.row0);
    bulk_commit_group();
  }
  e.count += 2;
}

// Load CNT chunks of the accumulator with back-to-back tcgen05.ld and one wait, optionally
// release them (arrive on `early_bar`) as soon as they are in registers, then store them.
template <int CNT, bool kRemote = false, bool kPeers = true>
__device__ __forceinline__ void epi_group(const GemmParams& p, EpiStage& e, uint32_t acc_t,
                                          const int (&cs)[CNT], int row, int col_base,
                                          uint32_t early_bar) {
  uint32_t r[CNT][32];
#pragma unroll
  for (int g = 0; g < CNT; ++g) tmem_ld_32x32b_x32(acc_t + cs[g] * 32, r[g]);
  tc_wait_ld();
  if (early_bar) {
    tc_fence_before();
    __syncwarp();
    if ((threadIdx.x & 31) == 0) {
      if (kRemote) mbar_arrive_cluster(early_bar);
      else mbar_arrive(early_bar);
    }
  }
  if constexpr (kPeers && CNT >= 2) {
    if (p.out_bf16 && p.tma_store && p.n_peers > 0 && cs[1] == cs[0] + 1) {
      stage_pair(p, e, r[0], r[1], col_base + cs[0] * 32);
      if constexpr (CNT == 3) stage_chunk<kPeers>(p, e, r[2], col_base + cs[2] * 32);
      return;
    }
  }
#pragma unroll
  for (int g = 0; g < CNT; ++g) {
    if (p.out_nvfp4) store_chunk_nvfp4(p, r[g], row, col_base + cs[g] * 32);
    else if (p.tma_store) stage_chunk<kPeers>(p, e, r[g], col_base + cs[g] * 32);
    else store_chunk(p, r[g], row, col_base + cs[g] * 32);
  }
}

// Drain a 256-column accumulator whose first (buffer 1) or last (buffer 0) OV chunks are
// shared with the other buffer: those chunks first, released on `early_bar` once they are in
// registers, then the rest.
template <int OV, bool kRemote, bool kPeers = true>
__device__ __forceinline__ void drain_overlapped(const GemmParams& p, EpiStage& e, uint32_t acc_t,
                                                 int b, int row, int col_base, uint32_t early_bar) {
  const int o = b ? 0 : 8 - OV;
  const int rest = b ? OV : 0;
  const int g0[3] = {o, o + 1, o + 2};
  if constexpr (OV == 3) {
    const int g1[3] = {rest, rest + 1, rest + 2}, g2[2] = {rest + 3, rest + 4};
    epi_group<3, kRemote, kPeers>(p, e, acc_t, g0, row, col_base, early_bar);
    epi_group<3, false, kPeers>(p, e, acc_t, g1, row, col_base, 0);
    epi_group<2, false, kPeers>(p, e, acc_t, g2, row, col_base, 0);
    return;
  }
  epi_group<3, false, kPeers>(p, e, acc_t, g0, row, col_base, 0);
  if constexpr (OV == 6) {
    const int g1[3] = {o + 3, o + 4, o + 5}, g2[2] = {rest, rest + 1};
    epi_group<3, kRemote, kPeers>(p, e, acc_t, g1, row, col_base, early_bar);
    epi_group<2, false, kPeers>(p, e, acc_t, g2, row, col_base, 0);
  } else if constexpr (OV == 5) {
    const int g1[2] = {o + 3, o + 4}, g2[2] = {rest, rest + 1}, g3[1] = {rest + 2};
    epi_group<2, kRemote, kPeers>(p, e, acc_t, g1, row, col_base, early_bar);
    epi_group<2, false, kPeers>(p, e, acc_t, g2, row, col_base, 0);
    epi_group<1, false, kPeers>(p, e, acc_t, g3, row, col_base, 0);
  } else {
    const int g1[1] = {o + 3}, g2[2] = {rest, rest + 1}, g3[2] = {rest + 2, rest + 3};
    epi_group<1, kRemote, kPeers>(p, e, acc_t, g1, row, col_base, early_bar);
    epi_group<2, false, kPeers>(p, e, acc_t, g2, row, col_base, 0);
    epi_group<2, false, kPeers>(p, e, acc_t, g3, row, col_base, 0);
  }
}

__device__ __forceinline__ void tc_mma_mxf4nvf4_sp(uint32_t d_tmem, uint64_t a_desc, uint64_t b_desc,
                                                   uint32_t meta_tmem, uint32_t idesc, uint32_t sfa_tmem,
                                                   uint32_t sfb_tmem, uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\tsetp.ne.b32 p, %7, 0;\n\t"
      "tcgen05.mma.sp.cta_group::1.kind::mxf4nvf4.block_scale.scale_vec::4X "
      "[%0], %1, %2, [%3], %4, [%5], [%6], p;\n\t}" ::"r"(d_tmem),
      "l"(a_desc), "l"(b_desc), "r"(meta_tmem), "r"(idesc), "r"(sfa_tmem), "r"(sfb_tmem),
      "r"(accumulate)
      : "memory");
}

template <int BN, bool SP = false, bool PEERS = false>
__global__ void __launch_bounds__(kNumThreads, 1)
    gemm_mxf4nvf4_kernel(const __grid_constant__ CUtensorMap tmap_a,
                         const __grid_constant__ CUtensorMap tmap_b,
                         const __grid_constant__ CUtensorMap tmap_c, const GemmParams p) {
  using C = Cfg<BN, SP>;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) &
                                             ~uintptr_t(1023));
  uint8_t* sA = smem;
  uint8_t* sB = sA + C::kStages * C::kABytes;
  uint8_t* sC = sB + C::kStages * C::kBBytes;  // 1024-aligned: stages are multiples of 1 KB
  uint8_t* sSfb = sC + C::kCBytes;
  uint64_t* bars = reinterpret_cast<uint64_t*>(sSfb + C::kSfbBytes);
  uint64_t* full = bars;                // A/B bytes + producer + the stage's 4 scale writers
  uint64_t* empty = bars + C::kStages;  // smem stage consumed
  uint64_t* acc_full = empty + C::kStages;
  uint64_t* acc_empty = acc_full + 2;
  uint64_t* acc_early = acc_full + 4;
  uint64_t* drain = acc_full + 6;
  uint64_t* sfb_full = drain + 1;       // dense: the stage's B scale atoms landed
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(sfb_full + C::kStages);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;

  if (threadIdx.x == 0) {
    for (int s = 0; s < C::kStages; ++s) {
      mbar_init(smem_u32(&full[s]), 1 + 4);
      mbar_init(smem_u32(&empty[s]), 1);
    }
    for (int b = 0; b < 2; ++b) {
      mbar_init(smem_u32(&acc_full[b]), 1);
      mbar_init(smem_u32(&acc_empty[b]), 4);
      mbar_init(smem_u32(&acc_early[b]), 4);
    }
    mbar_init(smem_u32(drain), 1);
    for (int s = 0; s < C::kStages; ++s) mbar_init(smem_u32(&sfb_full[s]), 1);
    *abort_flag = 0;
    fence_mbar_init();
    prefetch_tmap(&tmap_a);
    prefetch_tmap(&tmap_b);
    if (p.tma_store) prefetch_tmap(&tmap_c);
  }
  if (warp == 1) {
    tmem_alloc(smem_u32(tmem_slot), kTmemCols);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem_base = *tmem_slot;
  // Launched with programmatic stream serialization: the set-up above (barriers, TMEM,
  // descriptor prefetch) overlaps the tail of the previous kernel on the stream, typically the
  // scale reorder or the quantiser that wrote this GEMM's operands. No thread touches global
  // memory before that kernel has completed and its writes are visible.
  asm volatile("griddepcontrol.wait;" ::: "memory");

  if (warp == 0) {
    // ------------------------------------------------------------------ TMA producer
    if (lane == 0) {
      int it = 0;  // global stage counter across tiles
      bool ok = true;
      for (int t = blockIdx.x; t < p.num_tiles && ok; t += gridDim.x) {
        int tm, tn;
        tile_coords(p, t, tm, tn);
        const int m0 = tm * kBM, n0 = tn * BN;
        for (int kt = 0; kt < p.num_kt; ++kt, ++it) {
          const int s = it % C::kStages;
          const uint32_t j = static_cast<uint32_t>(it / C::kStages);
          if (!mbar_wait(smem_u32(&empty[s]), (j & 1u) ^ 1u, abort_flag, p.err_word,
                         kErrWaitSmemEmpty)) {
            ok = false;
            break;
          }
          const uint32_t fb = smem_u32(&full[s]);
          mbar_arrive_expect_tx(fb, C::kABytes + C::kBBytes);
          tma_load_2d(smem_u32(sA + s * C::kABytes), &tmap_a, kt * (SP ? 64 : kBKBytes), m0, fb);
          tma_load_2d(smem_u32(sB + s * C::kBBytes), &tmap_b, kt * kBKBytes, n0, fb);
          {
            // The stage's B scale atoms: per 128-row block of B one contiguous run of nkb atoms
            // (tcgen05 layout), to shared memory at (row block * atoms per stage + atom) * 512.
            // Row blocks past the end of B are not copied (the writers store zero scales).
            constexpr int kAps = C::kSfbAtomsPerStage;
            int nkb = p.ka - kt * kAps;
            if (nkb > kAps) nkb = kAps;
            int nrb = p.sfb_rowblocks - tn * (BN / 128);
            if (nrb > BN / 128) nrb = BN / 128;
            const uint32_t db = smem_u32(&sfb_full[s]);
            mbar_arrive_expect_tx(db, static_cast<uint32_t>(nrb * nkb * 512));
            for (int jb = 0; jb < nrb; ++jb)
              bulk_load(smem_u32(sSfb + s * C::kSfbStageBytes + jb * kAps * 512),
                        p.sfb + (static_cast<size_t>(tn * (BN / 128) + jb) * p.ka + kt * kAps) * 512,
                        static_cast<uint32_t>(nkb * 512), db);
          }
        }
      }
      if (!ok) {
        // Drain: the most recent fill of every stage must land before the CTA exits. "full"
        // also counts the scale writers, which may have left early; the bounded wait then
        // gives the copies far longer than they take.
        for (int back = 1; back <= C::kStages && it - back >= 0; ++back) {
          const int f = it - back;
          mbar_wait_drain(smem_u32(&full[f % C::kStages]),
                          static_cast<uint32_t>(f / C::kStages) & 1u, p.err_word);
          mbar_wait_drain(smem_u32(&sfb_full[f % C::kStages]),
                            static_cast<uint32_t>(f / C::kStages) & 1u, p.err_word);
        }
      }
    }
  } else if (warp == 1) {
    // ------------------------------------------------------------------ MMA issuer
    if (lane == 0) {
      const uint32_t idesc = make_idesc_mxf4nvf4(kBM, BN) | (SP ? (1u << 2) : 0u);  // bit 2: sparse A
      int it = 0;   // stage counter (also the position in the scale slot ring)
      int local = 0;
      bool ok = true;
      bool issued = false;
      for (int t = blockIdx.x; t < p.num_tiles && ok; t += gridDim.x, ++local) {
        const int b = local & 1;
        const uint32_t u = static_cast<uint32_t>(local >> 1);
        if (!mbar_wait(smem_u32(&acc_empty[b]), (u & 1u) ^ 1u, abort_flag, p.err_word,
                       kErrWaitAccEmpty)) {
          ok = false;
          break;
        }
        if (C::kOverlap && local > 0) {
          const uint32_t up = static_cast<uint32_t>((local - 1) >> 1);
          if (!mbar_wait(smem_u32(&acc_early[b ^ 1]), up & 1u, abort_flag, p.err_word,
                         kErrWaitAccEmpty)) {
            ok = false;
            break;
          }
        }
        tc_fence_after();
        const uint32_t acc_t = tmem_base + (b ? C::kAccBase1 : 0);
        for (int kt = 0; kt < p.num_kt && ok; ++kt, ++it) {
          const int s = it % C::kStages;
          const uint32_t j = static_cast<uint32_t>(it / C::kStages);
          // One spin-wait per stage: A/B bytes, producer and the stage's scale writers.
          if (!mbar_spin_wait<false>(smem_u32(&full[s]), j & 1u, abort_flag, p.err_word,
                                     kErrWaitTmaFull)) {
            ok = false;
            break;
          }
          tc_fence_after();
          const int slot = it % C::kSfSlots;
          if constexpr (SP) {
            // Two sparse MMAs (128 logical K each): compressed A 32 bytes (+2 descriptor units)
            // and B 64 bytes (+4) apart; scales one word per row (SFA at +4m, SFB at +8m),
            // metadata two columns per MMA at +32 in the rows' own lanes.
            int nm = p.ka - kt * 2;
            if (nm > 2) nm = 2;
            const uint64_t ad0 = make_sdesc(smem_u32(sA + s * C::kABytes), 16, 512, 4);
            const uint64_t bd0 = make_sdesc(smem_u32(sB + s * C::kBBytes), 16, 1024, 2);
            const uint32_t sf_t = tmem_base + C::kSfCol + slot * kSfSlotCols;
            for (int m = 0; m < nm; ++m)
              tc_mma_mxf4nvf4_sp(acc_t, ad0 + 2 * m, bd0 + 4 * m, sf_t + 32 + 2 * m, idesc,
                                 sf_t + 4 * m, sf_t + kSfbOff + 8 * m, (kt > 0 || m > 0) ? 1u : 0u);
          } else {
            int nkb = p.ka - kt * kKBlocksPerStage;
            if (nkb > kKBlocksPerStage) nkb = kKBlocksPerStage;
            // Descriptor start addresses are in 16-byte units: +2 per 32-byte K-block.
            const uint64_t ad0 = make_sdesc(smem_u32(sA + s * C::kABytes), 16, 1024, 2);
            const uint64_t bd0 = make_sdesc(smem_u32(sB + s * C::kBBytes), 16, 1024, 2);
            const uint32_t sf_t = tmem_base + C::kSfCol + slot * kSfSlotCols;
            if (nkb == kKBlocksPerStage) {
#pragma unroll
              for (int kb = 0; kb < kKBlocksPerStage; ++kb)
                tc_mma_mxf4nvf4(acc_t, ad0 + 2 * kb, bd0 + 2 * kb, idesc, sf_t + kb * 4,
                                sf_t + kSfbOff + kb * C::kSfbColsPerKb, (kt > 0 || kb > 0) ? 1u : 0u);
            } else {
              for (int kb = 0; kb < nkb; ++kb)
                tc_mma_mxf4nvf4(acc_t, ad0 + 2 * kb, bd0 + 2 * kb, idesc, sf_t + kb * 4,
                                sf_t + kSfbOff + kb * C::kSfbColsPerKb, (kt > 0 || kb > 0) ? 1u : 0u);
            }
          }
          issued = true;
          // One commit frees both the smem stage and its TMEM scale slot: the writers of a
          // slot wait on "empty" of the stage that used it last (a second commit per stage
          // costs about 60 cycles of MMA issue).
          tc_commit(smem_u32(&empty[s]));
        }
        if (!ok) break;
        tc_commit(smem_u32(&acc_full[b]));
      }
      if (!ok && issued) {
        tc_commit(smem_u32(drain));
        mbar_wait_drain(smem_u32(drain), 0, p.err_word);
      }
    }
  } else if (warp >= 6) {
    // ------------------------------------------------------------------ scale writers
    // In an atom, lane l's 16 bytes are 4 words; word g holds the 4 K-scales of row 32g + l.
    // Each writer reads its lanes' words of the stage's atoms straight from global memory (L2)
    // into registers, so scales take no shared memory and no copy of their own. Slot columns:
    // SFA K-block kb's words at +4*kb, SFB atom jb of K-block kb at +16 + kb*(4*atoms) + 4*jb.
    // K-blocks past the end of K and atoms past the last row block are written as zero
    // scales; no output the kernel stores depends on them.
    const int q = warp & 3;
    const int wgroup = (warp - 6) >> 2;
    const uint32_t lane_base = tmem_base + (static_cast<uint32_t>(q * 32) << 16);
    int it = 0;
    bool ok = true;
    for (int t = blockIdx.x; t < p.num_tiles && ok; t += gridDim.x) {
      int tm, tn;
      tile_coords(p, t, tm, tn);
      const uint8_t* ga = p.sfa + static_cast<size_t>(tm) * p.ka * 512 + lane * 16;
      if (wgroup == 0) {
        // The tile's A scale atoms (ka x 512 bytes) into L2 at once, quadrant q taking every
        // fourth 128-byte line, so that the per-stage loads below wait for L2, not DRAM, on
        // the first tiles after the operands were written or evicted.
        const uint8_t* row_block = p.sfa + static_cast<size_t>(tm) * p.ka * 512;
        for (int l = q * 32 + lane; l < p.ka * 4; l += 128)
          asm volatile("prefetch.global.L2 [%0];" ::"l"(row_block + static_cast<size_t>(l) * 128));
      }
      for (int kt = 0; kt < p.num_kt && ok; ++kt, ++it) {
        if ((it % kWriterGroups) != wgroup) continue;
        const int s = it % C::kStages;
        const int slot = it % C::kSfSlots;
        int nkb = p.ka - kt * kKBlocksPerStage;
        if (nkb > kKBlocksPerStage) nkb = kKBlocksPerStage;
        // SFA: only word q of each atom row (the 4 K-scales of row 32q + lane) is read by the
        // MMA rows of quadrant q, so each writer stores that one column per K-block. SFB rows
        // map to accumulator columns, which every quadrant computes: all four words, in every
        // quadrant.
        uint32_t va[kKBlocksPerStage], vb[4 * C::kSfbColsPerKb], vm[4];
        if constexpr (SP) {
          // Per sparse MMA m (atom kt*2 + m, 128 logical K): SFA word q, SFB all of both row
          // blocks' words, metadata words 2m, 2m+1 of this row (8 bytes = 16 groups).
          int nm = p.ka - kt * 2;
          if (nm > 2) nm = 2;
          const int row = tm * kBM + q * 32 + lane;
          const uint8_t* gm = p.meta + static_cast<size_t>(row < p.M ? row : 0) * (p.K / 16) + kt * 16;
#pragma unroll
          for (int m = 0; m < 2; ++m) {
            const bool in = m < nm;
            va[m] = in ? __ldg(reinterpret_cast<const uint32_t*>(ga + q * 4 + (kt * 2 + m) * 512)) : 0u;
#pragma unroll
            for (int h = 0; h < 2; ++h)
              vm[2 * m + h] = (in && row < p.M) ? __ldg(reinterpret_cast<const uint32_t*>(gm + 8 * m + 4 * h)) : 0u;
          }
          // B scales from the stage's shared-memory copy (see the dense branch).
          if (!mbar_wait(smem_u32(&sfb_full[s]), static_cast<uint32_t>(it / C::kStages) & 1u,
                         abort_flag, p.err_word, kErrWaitSfFull)) {
            ok = false;
            break;
          }
          const uint4* sbs = reinterpret_cast<const uint4*>(sSfb + s * C::kSfbStageBytes);
#pragma unroll
          for (int m = 0; m < 2; ++m) {
#pragma unroll
            for (int jb = 0; jb < C::kSfbAtoms; ++jb) {
              const int rb = tn * (BN / 128) + jb;
              uint4 x = make_uint4(0u, 0u, 0u, 0u);
              if (m < nm && rb < p.sfb_rowblocks) x = sbs[(jb * 2 + m) * 32 + lane];
              const int o = m * 8 + 4 * jb;
              vb[o + 0] = x.x; vb[o + 1] = x.y; vb[o + 2] = x.z; vb[o + 3] = x.w;
            }
          }
        } else {
#pragma unroll
        for (int kb = 0; kb < kKBlocksPerStage; ++kb) {
          va[kb] = 0u;
          if (kb < nkb)
            va[kb] = __ldg(reinterpret_cast<const uint32_t*>(ga + q * 4 + (kt * kKBlocksPerStage + kb) * 512));
        }
        // B scales from the stage's shared-memory copy (one bulk copy per CTA and stage,
        // instead of the same 4 KB loaded from L2 by each of the four quadrant writers).
        if (!mbar_wait(smem_u32(&sfb_full[s]), static_cast<uint32_t>(it / C::kStages) & 1u,
                       abort_flag, p.err_word, kErrWaitSfFull)) {
          ok = false;
          break;
        }
        const uint4* sb = reinterpret_cast<const uint4*>(sSfb + s * C::kSfbStageBytes);
#pragma unroll
        for (int kb = 0; kb < kKBlocksPerStage; ++kb) {
#pragma unroll
          for (int jb = 0; jb < C::kSfbAtoms; ++jb) {
            const int rb = tn * (BN / 128) + jb;
            uint4 x = make_uint4(0u, 0u, 0u, 0u);
            if (kb < nkb && rb < p.sfb_rowblocks) x = sb[(jb * kKBlocksPerStage + kb) * 32 + lane];
            const int o = kb * C::kSfbColsPerKb + 4 * jb;
            vb[o + 0] = x.x; vb[o + 1] = x.y; vb[o + 2] = x.z; vb[o + 3] = x.w;
          }
        }
        }
        // The slot's previous use (stage u = it - kSfSlots) must have been consumed: wait for
        // phase u / kStages of that stage's "empty". That barrier cannot be a phase further on,
        // since its next phase needs the MMAs of stage u + kStages > it, which wait for this
        // writer. This also orders the "full" arrival below after that barrier's previous
        // phase, because kSfSlots <= kStages.
        if (it >= C::kSfSlots) {
          const int u = it - C::kSfSlots;
          if (!mbar_wait(smem_u32(&empty[u % C::kStages]),
                         static_cast<uint32_t>(u / C::kStages) & 1u, abort_flag, p.err_word,
                         kErrWaitSfEmpty)) {
            ok = false;
            break;
          }
        }
        tc_fence_after();
        const uint32_t sf_t = lane_base + C::kSfCol + slot * kSfSlotCols;
        if constexpr (SP) {
#pragma unroll
          for (int m = 0; m < 2; ++m) tmem_st_32x32b_x1(sf_t + 4 * m + q, va[m]);
          tmem_st_32x32b_x16(sf_t + kSfbOff, vb);
          tmem_st_32x32b_x4(sf_t + 32, vm[0], vm[1], vm[2], vm[3]);
        } else {
#pragma unroll
          for (int kb = 0; kb < kKBlocksPerStage; ++kb) tmem_st_32x32b_x1(sf_t + kb * 4 + q, va[kb]);
          tmem_st_32x32b_x16(sf_t + kSfbOff, vb);
          if (C::kSfbAtoms == 2) tmem_st_32x32b_x16(sf_t + kSfbOff + 16, vb + 16);
        }
        tc_wait_st();
        tc_fence_before();
        __syncwarp();
        if (lane == 0) mbar_arrive(smem_u32(&full[s]));
      }
    }
  } else {
    // ------------------------------------------------------------------ epilogue
    const int q = warp & 3;                 // TMEM lane quadrant of this warp
    const int row_in_tile = q * 32 + lane;
    EpiStage e{sC + (warp - 2) * C::kCBufBytes, 0u, &tmap_c, 0};
    int local = 0;
    for (int t = blockIdx.x; t < p.num_tiles; t += gridDim.x, ++local) {
      const int b = local & 1;
      const uint32_t u = static_cast<uint32_t>(local >> 1);
      if (!mbar_wait(smem_u32(&acc_full[b]), u & 1u, abort_flag, p.err_word, kErrWaitAccFull))
        break;
      tc_fence_after();
      int tm, tn;
      tile_coords(p, t, tm, tn);
      const int row = tm * kBM + row_in_tile;
      const int col_base = tn * BN;
      e.row0 = tm * kBM + q * 32;
      const uint32_t acc_t = tmem_base + (static_cast<uint32_t>(q * 32) << 16) +
                             (b ? C::kAccBase1 : 0);
      if (C::kOverlap) {
        // The columns shared with the other buffer: buffer 0's chunks 3..7, buffer 1's
        // chunks 0..4. Load them first and release them as soon as they are in registers.
        drain_overlapped<C::kOverlapChunks, false, PEERS>(p, e, acc_t, b, row, col_base,
                                                   smem_u32(&acc_early[b]));
      } else {
#pragma unroll
        for (int c = 0; c < C::kChunks; c += 2) {
          const int g[2] = {c, c + 1};
          epi_group<2, false, PEERS>(p, e, acc_t, g, row, col_base, 0);
        }
      }
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(smem_u32(&acc_empty[b]));
    }
    if (lane == 0) {
      bulk_wait_group<0>();  // stores complete before the CTA's smem goes away
      if (PEERS && p.n_peers) fence_sc_sys();  // and, for peer destinations, visible system-wide
    }
    __syncwarp();
  }

  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  if (warp == 1) tmem_dealloc(tmem_base, kTmemCols);
}


// ---- pair-wise 2:4 sparse variant (gemm_mxf4nvf4_kernel<256, true>) --------------------
// A is stored compressed ([M][K/4] bytes: the 2 kept pairs of every group of 8 K elements) with
// pair metadata [M][K/16] (a nibble per group: first kept pair | second << 2) and UE4M3 scales
// per 32 K elements (A and B); B is dense. One sparse MMA covers 128 logical K (32 compressed
// bytes of A, 64 bytes of B); a stage is 256 logical K: A 8 KB (one 64-byte-wide, 64-byte-
// swizzled box) + B 32 KB, two MMAs of 128 x 256, four stages - the dense 128 x 256 kernel's
// structure, tile order, epilogue and accumulator overlap. Per row and per MMA the MMA reads
// one word of A scales and one of B scales (byte j for logical K 32j..32j+31) and two TMEM
// columns of metadata in the row's own lane (measured on B200 with one-hot probes); the writers
// load them from L2 and store SFA diagonally, SFB whole and the metadata at slot column +32.

// ---- SM-pair kernel (cta_group::2): 256 x 256 tiles ------------------------------------
// The two CTAs of a cluster work on one 256 x 256 output tile. Each loads its own 128 rows
// of A and its own 128 rows of B (so each SM moves half the B bytes of the one-SM kernel)
// plus the scales for its A rows and for all 256 B rows. The leader (rank 0) issues
// M=256 x N=256 x K=64 MMAs that read both CTAs' shared memory and write each CTA's TMEM
// (its 128 rows x 256 columns); both CTAs run scale writers and an epilogue for their own
// TMEM. Barriers that gather both CTAs live in the leader: "full" (both CTAs' A/B byte
// counts through TMA with .cta_group::2 plus both CTAs' scale writers, 1 + 8 arrivals) and the
// accumulator releases ("acc_empty", "acc_early", 8 arrivals); the leader's commits signal
// each CTA's own "empty" (stage and scale slot) and "acc_full" by address.
struct PairCfg {
  static constexpr int kABytes = 128 * kBKBytes;       // this CTA's 128 rows of A
  static constexpr int kBBytes = 128 * kBKBytes;       // this CTA's 128 rows of B
  static constexpr int kStageBytes = kABytes + kBBytes;  // 32 KB; scales bypass smem
  static constexpr int kStages = 6;
  static constexpr int kCBufBytes = 32 * 32 * 4;
  static constexpr int kCBytes = 4 * 2 * kCBufBytes;
  static constexpr int kBarBytes = 512;
  static constexpr int kSmemBytes = 1024 + kStages * kStageBytes + kCBytes + kBarBytes;
  static constexpr int kSfSlots = NVFP4_PAIR_SF_SLOTS;  // ring of per-stage scale slots
  static constexpr int kSfCol = kTmemCols - kSfSlots * kSfSlotCols;
  static constexpr int kAccBase1 = kSfCol - 256;       // as in the one-SM N=256 kernel
  static constexpr int kOverlapChunks = (256 - kAccBase1 + 31) / 32;
  static_assert(kSmemBytes <= 232448, "shared memory budget");
  static_assert(kSfSlots <= kStages, "a writer's slot wait must also order its full[] arrival");
};

__global__ void __launch_bounds__(kNumThreads, 1)
    gemm_mxf4nvf4_pair_kernel(const __grid_constant__ CUtensorMap tmap_a,
                              const __grid_constant__ CUtensorMap tmap_b,
                              const __grid_constant__ CUtensorMap tmap_c, const GemmParams p) {
  using C = PairCfg;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) &
                                             ~uintptr_t(1023));
  uint8_t* sA = smem;
  uint8_t* sB = sA + C::kStages * C::kABytes;
  uint8_t* sC = sB + C::kStages * C::kBBytes;
  uint64_t* bars = reinterpret_cast<uint64_t*>(sC + C::kCBytes);
  uint64_t* full = bars;                    // leader: A/B bytes of both CTAs
  uint64_t* empty = full + C::kStages;      // each CTA: stage consumed
  uint64_t* acc_full = empty + C::kStages;
  uint64_t* acc_empty = acc_full + 2;       // leader, 8 arrivals
  uint64_t* acc_early = acc_full + 4;       // leader, 8 arrivals
  uint64_t* drain = acc_full + 6;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(drain + 1);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const uint32_t rank = cluster_ctarank();
  const int cid = blockIdx.x >> 1, ncl = gridDim.x >> 1;
  auto to_leader = [](const uint64_t* b) { return mapa_shared(smem_u32(b), 0); };
  auto to_peer = [](const uint64_t* b) { return mapa_shared(smem_u32(b), 1); };

  if (threadIdx.x == 0) {
    for (int s = 0; s < C::kStages; ++s) {
      mbar_init(smem_u32(&full[s]), 1 + 8);  // leader's expect_tx + both CTAs' scale writers
      mbar_init(smem_u32(&empty[s]), 1);
    }
    for (int b = 0; b < 2; ++b) {
      mbar_init(smem_u32(&acc_full[b]), 1);
      mbar_init(smem_u32(&acc_empty[b]), 8);
      mbar_init(smem_u32(&acc_early[b]), 8);
    }
    mbar_init(smem_u32(drain), 1);
    *abort_flag = 0;
    fence_mbar_init();
    prefetch_tmap(&tmap_a);
    prefetch_tmap(&tmap_b);
    if (p.tma_store) prefetch_tmap(&tmap_c);
  }
  if (warp == 1) {
    tmem_alloc_pair(smem_u32(tmem_slot), kTmemCols);
    tmem_relinquish_pair();
  }
  tc_fence_before();
  __syncthreads();
  cluster_sync();  // the peer's barriers exist before any cross-CTA arrival or byte count
  tc_fence_after();
  const uint32_t tmem_base = *tmem_slot;

  if (warp == 0) {
    // ------------------------------------------------------------------ TMA producer (both)
    if (lane == 0) {
      const uint32_t full_l0 = to_leader(&full[0]);
      int it = 0;
      bool ok = true;
      for (int t = cid; t < p.num_tiles && ok; t += ncl) {
        int tm, tn;
        tile_coords(p, t, tm, tn);
        const int m0 = tm * 256 + static_cast<int>(rank) * 128, n0 = tn * 256;
        for (int kt = 0; kt < p.num_kt; ++kt, ++it) {
          const int s = it % C::kStages;
          const uint32_t j = static_cast<uint32_t>(it / C::kStages);
          if (!mbar_wait_cluster(smem_u32(&empty[s]), (j & 1u) ^ 1u, abort_flag, p.err_word,
                                 kErrWaitSmemEmpty)) {
            ok = false;
            break;
          }
          if (rank == 0) mbar_arrive_expect_tx(smem_u32(&full[s]), 2 * (C::kABytes + C::kBBytes));
          const uint32_t fb = full_l0 + s * 8;
          tma_load_2d_pair(smem_u32(sA + s * C::kABytes), &tmap_a, kt * kBKBytes, m0, fb);
          tma_load_2d_pair(smem_u32(sB + s * C::kBBytes), &tmap_b, kt * kBKBytes,
                           n0 + static_cast<int>(rank) * 128, fb);
        }
      }
      if (!ok) {
        // The leader's "full" counts both CTAs' bytes (and the scale writers, which may have
        // left early: the bounded wait then gives the copies far longer than they take); the
        // closing cluster barrier keeps the peer resident until it returns.
        for (int back = 1; back <= C::kStages && it - back >= 0; ++back) {
          const int f = it - back;
          if (rank == 0)
            mbar_wait_drain(smem_u32(&full[f % C::kStages]),
                            static_cast<uint32_t>(f / C::kStages) & 1u, p.err_word);
        }
      }
    }
  } else if (warp == 1) {
    // ------------------------------------------------------------------ MMA issuer (leader)
    if (lane == 0 && rank == 0) {
      const uint32_t idesc = make_idesc_mxf4nvf4(256, 256);
      int it = 0, local = 0;
      bool ok = true, issued = false;
      for (int t = cid; t < p.num_tiles && ok; t += ncl, ++local) {
        const int b = local & 1;
        const uint32_t u = static_cast<uint32_t>(local >> 1);
        if (!mbar_wait_cluster(smem_u32(&acc_empty[b]), (u & 1u) ^ 1u, abort_flag, p.err_word,
                               kErrWaitAccEmpty)) {
          ok = false;
          break;
        }
        if (local > 0) {
          const uint32_t up = static_cast<uint32_t>((local - 1) >> 1);
          if (!mbar_wait_cluster(smem_u32(&acc_early[b ^ 1]), up & 1u, abort_flag, p.err_word,
                                 kErrWaitAccEmpty)) {
            ok = false;
            break;
          }
        }
        tc_fence_after();
        const uint32_t acc_t = tmem_base + (b ? C::kAccBase1 : 0);
        for (int kt = 0; kt < p.num_kt && ok; ++kt, ++it) {
          const int s = it % C::kStages;
          const uint32_t j = static_cast<uint32_t>(it / C::kStages);
          // One spin-wait per stage: both CTAs' A/B bytes and both CTAs' scale writers.
          if (!mbar_spin_wait<true>(smem_u32(&full[s]), j & 1u, abort_flag, p.err_word,
                                    kErrWaitTmaFull)) {
            ok = false;
            break;
          }
          const int slot = it % C::kSfSlots;
          tc_fence_after();
          int nkb = p.ka - kt * kKBlocksPerStage;
          if (nkb > kKBlocksPerStage) nkb = kKBlocksPerStage;
          const uint64_t ad0 = make_sdesc(smem_u32(sA + s * C::kABytes), 16, 1024, 2);
          const uint64_t bd0 = make_sdesc(smem_u32(sB + s * C::kBBytes), 16, 1024, 2);
          const uint32_t sf_t = tmem_base + C::kSfCol + slot * kSfSlotCols;
          if (nkb == kKBlocksPerStage) {
#pragma unroll
            for (int kb = 0; kb < kKBlocksPerStage; ++kb)
              tc_mma_mxf4nvf4_pair(acc_t, ad0 + 2 * kb, bd0 + 2 * kb, idesc, sf_t + kb * 4,
                                   sf_t + kSfbOff + kb * 8, (kt > 0 || kb > 0) ? 1u : 0u);
          } else {
            for (int kb = 0; kb < nkb; ++kb)
              tc_mma_mxf4nvf4_pair(acc_t, ad0 + 2 * kb, bd0 + 2 * kb, idesc, sf_t + kb * 4,
                                   sf_t + kSfbOff + kb * 8, (kt > 0 || kb > 0) ? 1u : 0u);
          }
          issued = true;
          // "empty" also frees the stage's TMEM scale slot in both CTAs.
          tc_commit_pair(smem_u32(&empty[s]));
          tc_commit_pair(to_peer(&empty[s]));
        }
        if (!ok) break;
        tc_commit_pair(smem_u32(&acc_full[b]));
        tc_commit_pair(to_peer(&acc_full[b]));
      }
      if (!ok && issued) {
        tc_commit_pair(smem_u32(drain));
        mbar_wait_drain(smem_u32(drain), 0, p.err_word);
      }
    }
  } else if (warp >= 6) {
    // ------------------------------------------------------------------ scale writers (both)
    const int q = warp & 3;
    const int wgroup = (warp - 6) >> 2;
    const uint32_t lane_base = tmem_base + (static_cast<uint32_t>(q * 32) << 16);
    const uint32_t full_l0 = to_leader(&full[0]);
    int it = 0;
    bool ok = true;
    for (int t = cid; t < p.num_tiles && ok; t += ncl) {
      int tm, tn;
      tile_coords(p, t, tm, tn);
      const int ra = tm * 2 + static_cast<int>(rank);  // 128-row blocks
      const int rb0 = tn * 2;
      for (int kt = 0; kt < p.num_kt && ok; ++kt, ++it) {
        if ((it % kWriterGroups) != wgroup) continue;
        const int s = it % C::kStages;
        const int slot = it % C::kSfSlots;
        int nkb = p.ka - kt * kKBlocksPerStage;
        if (nkb > kKBlocksPerStage) nkb = kKBlocksPerStage;
        // This CTA's 128 rows of A (word q only: see the one-SM kernel) and all 256 rows of B,
        // straight from global memory (L2).
        uint32_t va[kKBlocksPerStage], vb[32];
#pragma unroll
        for (int kb = 0; kb < kKBlocksPerStage; ++kb) {
          va[kb] = 0u;
          if (kb < nkb && ra < p.sfa_rowblocks)
            va[kb] = __ldg(reinterpret_cast<const uint32_t*>(
                p.sfa + (static_cast<size_t>(ra) * p.ka + kt * kKBlocksPerStage + kb) * 512 +
                lane * 16 + q * 4));
#pragma unroll
          for (int jb = 0; jb < 2; ++jb) {
            uint4 x = make_uint4(0u, 0u, 0u, 0u);
            if (kb < nkb && rb0 + jb < p.sfb_rowblocks)
              x = __ldg(reinterpret_cast<const uint4*>(
                  p.sfb + (static_cast<size_t>(rb0 + jb) * p.ka + kt * kKBlocksPerStage + kb) * 512 +
                  lane * 16));
            const int o = kb * 8 + 4 * jb;
            vb[o + 0] = x.x; vb[o + 1] = x.y; vb[o + 2] = x.z; vb[o + 3] = x.w;
          }
        }
        // The slot's previous use (stage u = it - kSfSlots) must have been consumed: phase
        // u / kStages of this CTA's "empty" for that stage (it cannot be a phase further on,
        // whose MMAs wait for this writer). Because kSfSlots <= kStages this also orders the
        // arrival below after the leader's "full" barrier finished its previous phase.
        if (it >= C::kSfSlots) {
          const int u = it - C::kSfSlots;
          if (!mbar_wait_cluster(smem_u32(&empty[u % C::kStages]),
                                 static_cast<uint32_t>(u / C::kStages) & 1u, abort_flag,
                                 p.err_word, kErrWaitSfEmpty)) {
            ok = false;
            break;
          }
        }
        tc_fence_after();
        const uint32_t sf_t = lane_base + C::kSfCol + slot * kSfSlotCols;
#pragma unroll
        for (int kb = 0; kb < kKBlocksPerStage; ++kb) tmem_st_32x32b_x1(sf_t + kb * 4 + q, va[kb]);
        tmem_st_32x32b_x16(sf_t + kSfbOff, vb);
        tmem_st_32x32b_x16(sf_t + kSfbOff + 16, vb + 16);
        tc_wait_st();
        tc_fence_before();
        __syncwarp();
        if (lane == 0) mbar_arrive_cluster(full_l0 + s * 8);
      }
    }
  } else {
    // ------------------------------------------------------------------ epilogue (both)
    const int q = warp & 3;
    const int row_in_tile = static_cast<int>(rank) * 128 + q * 32 + lane;
    EpiStage e{sC + (warp - 2) * 2 * C::kCBufBytes, 0u, &tmap_c, 0};
    const uint32_t early_l0 = to_leader(&acc_early[0]);
    const uint32_t empty_l0 = to_leader(&acc_empty[0]);
    int local = 0;
    for (int t = cid; t < p.num_tiles; t += ncl, ++local) {
      const int b = local & 1;
      const uint32_t u = static_cast<uint32_t>(local >> 1);
      if (!mbar_wait_cluster(smem_u32(&acc_full[b]), u & 1u, abort_flag, p.err_word,
                             kErrWaitAccFull))
        break;
      tc_fence_after();
      int tm, tn;
      tile_coords(p, t, tm, tn);
      const int row = tm * 256 + row_in_tile;
      const int col_base = tn * 256;
      e.row0 = tm * 256 + static_cast<int>(rank) * 128 + q * 32;
      const uint32_t acc_t = tmem_base + (static_cast<uint32_t>(q * 32) << 16) +
                             (b ? C::kAccBase1 : 0);
      drain_overlapped<C::kOverlapChunks, true>(p, e, acc_t, b, row, col_base, early_l0 + b * 8);
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive_cluster(empty_l0 + b * 8);
    }
    if (lane == 0) {
      bulk_wait_group<0>();
      if (p.n_peers) fence_sc_sys();
    }
    __syncwarp();
  }

  tc_fence_before();
  __syncthreads();
  cluster_sync();  // the leader's MMAs into the peer's TMEM are complete on both sides
  tc_fence_after();
  if (warp == 1) tmem_dealloc_pair(tmem_base, kTmemCols);
}

// One CTA waits on an mbarrier nothing completes, with a short limit: exercises the
// timeout path (error word + clean return) without faulting or hanging the GPU.
__global__ void wait_selftest_kernel(uint64_t limit_ns, uint32_t* err_word) {
  __shared__ uint64_t bar;
  if (threadIdx.x == 0) {
    mbar_init(smem_u32(&bar), 1);
    fence_mbar_init();
    const uint64_t t0 = globaltimer_ns();
    while (!mbar_try_wait(smem_u32(&bar), 0)) {
      if (globaltimer_ns() - t0 > limit_ns) {
        atomicOr(err_word, kErrTest);
        break;
      }
    }
  }
}

// ---- host side ----------------------------------------------------------------------
using EncodeTiledFn = CUresult (*)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*,
                                   const cuuint64_t*, const cuuint64_t*, const cuuint32_t*,
                                   const cuuint32_t*, CUtensorMapInterleave, CUtensorMapSwizzle,
                                   CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

EncodeTiledFn get_encode_fn() {
  static EncodeTiledFn fn = nullptr;
  static std::once_flag once;
  std::call_once(once, [] {
    void* ptr = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPointByVersion("cuTensorMapEncodeTiled", &ptr, 12000,
                                         cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<EncodeTiledFn>(ptr);
  });
  return fn;
}

// Packed FP4 rows as a 2-D UINT8 tensor [rows][K/2], box {128 bytes, box_rows}, 128-byte
// swizzle, zero fill out of bounds.
// Packed operand [rows][K/2] bytes, K-major. sw64: a 64-byte-wide box with 64-byte swizzle (the
// sparse kernel's compressed A stage); otherwise 128 bytes with 128-byte swizzle.
bool encode_operand_map(CUtensorMap* map, const void* base, int rows, int K, int box_rows,
                        std::string* err, bool sw64 = false) {
  EncodeTiledFn enc = get_encode_fn();
  if (!enc) {
    set_err(err, "cuTensorMapEncodeTiled unavailable from the driver");
    return false;
  }
  cuuint64_t dims[2] = {static_cast<cuuint64_t>(K / 2), static_cast<cuuint64_t>(rows)};
  cuuint64_t strides[1] = {static_cast<cuuint64_t>(K / 2)};
  cuuint32_t box[2] = {static_cast<cuuint32_t>(sw64 ? 64 : kBKBytes), static_cast<cuuint32_t>(box_rows)};
  cuuint32_t estr[2] = {1, 1};
  CUresult r = enc(map, CU_TENSOR_MAP_DATA_TYPE_UINT8, 2, const_cast<void*>(base), dims, strides,
                   box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE,
                   sw64 ? CU_TENSOR_MAP_SWIZZLE_64B : CU_TENSOR_MAP_SWIZZLE_128B,
                   CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS) {
    set_err(err, "cuTensorMapEncodeTiled failed (code " + std::to_string(static_cast<int>(r)) + ")");
    return false;
  }
  return true;
}

// Row-major output [M][N] (row pitch `pitch` elements) as a 2-D tensor, box 32 x 32 elements, swizzled to match the
// epilogue's staging layout (64-byte rows for BF16, 128-byte rows for FP32).
bool encode_output_map(CUtensorMap* map, void* base, int M, int N, long pitch, bool bf16,
                       std::string* err, bool wide = false) {
  EncodeTiledFn enc = get_encode_fn();
  if (!enc) {
    set_err(err, "cuTensorMapEncodeTiled unavailable from the driver");
    return false;
  }
  const size_t es = bf16 ? 2 : 4;
  cuuint64_t dims[2] = {static_cast<cuuint64_t>(N), static_cast<cuuint64_t>(M)};
  cuuint64_t strides[1] = {static_cast<cuuint64_t>(pitch * es)};
  // wide (BF16 only): box 64 x 32, 128-byte rows, 128-byte swizzle.
  cuuint32_t box[2] = {wide ? 64u : 32u, 32};
  cuuint32_t estr[2] = {1, 1};
  CUresult r = enc(map, bf16 ? CU_TENSOR_MAP_DATA_TYPE_BFLOAT16 : CU_TENSOR_MAP_DATA_TYPE_FLOAT32, 2,
                   base, dims, strides, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE,
                   (bf16 && !wide) ? CU_TENSOR_MAP_SWIZZLE_64B : CU_TENSOR_MAP_SWIZZLE_128B,
                   CU_TENSOR_MAP_L2_PROMOTION_NONE, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS) {
    set_err(err, "cuTensorMapEncodeTiled (output) failed (code " + std::to_string(static_cast<int>(r)) + ")");
    return false;
  }
  return true;
}

// Small cache of encoded tensor maps: encoding is pure host work (a few microseconds per map)
// that would otherwise sit in front of every launch. A map depends only on the key below, so
// a hit is exact; entries are replaced round-robin.
struct MapKey {
  const void* base;
  long rows, cols;
  int box, kind;  // kind: 0 = operand, 1 = BF16 output, 2 = FP32 output, 3 = operand, 64-byte box
  long pitch = 0;  // outputs: row pitch in elements
  bool operator==(const MapKey& o) const {
    return base == o.base && rows == o.rows && cols == o.cols && box == o.box && kind == o.kind &&
           pitch == o.pitch;
  }
};
struct MapCache {
  static constexpr int kEntries = 64;
  MapKey key[kEntries];
  CUtensorMap map[kEntries];
  bool used[kEntries] = {};
  int next = 0;
  std::mutex mu;
};
MapCache g_maps;

bool cached_map(const MapKey& k, CUtensorMap* out, std::string* err) {
  {
    std::lock_guard<std::mutex> lk(g_maps.mu);
    for (int i = 0; i < MapCache::kEntries; ++i)
      if (g_maps.used[i] && g_maps.key[i] == k) {
        *out = g_maps.map[i];
        return true;
      }
  }
  bool ok = (k.kind == 0 || k.kind == 3)
                ? encode_operand_map(out, k.base, static_cast<int>(k.rows), static_cast<int>(k.cols),
                                     k.box, err, k.kind == 3)
                        : encode_output_map(out, const_cast<void*>(k.base), static_cast<int>(k.rows),
                                            static_cast<int>(k.cols), k.pitch, k.kind == 1, err);
  if (!ok) return false;
  std::lock_guard<std::mutex> lk(g_maps.mu);
  const int i = g_maps.next;
  g_maps.next = (i + 1) % MapCache::kEntries;
  g_maps.key[i] = k;
  g_maps.map[i] = *out;
  g_maps.used[i] = true;
  return true;
}

struct DeviceState {
  bool init = false;
  int sms = 0;
  int cc_major = 0, cc_minor = 0;
  bool attr_set[6] = {};  // one-SM kernels: [128, 256, sparse] x [no peers, peers]
  bool pair_attr_set = false;
  int pair_clusters = 0;  // co-resident SM-pair clusters of the pair kernel
  uint32_t* err_word = nullptr;
  // Workspaces for canonical -> tcgen05 scale reordering, one per stream (grown on demand):
  // calls on different streams never share reordered scales, and calls on one stream are
  // ordered by the stream itself.
  struct Workspace {
    cudaStream_t stream;
    uint8_t* ptr;
    size_t bytes;
  };
  std::vector<Workspace> ws;
};

std::mutex g_mu;
std::vector<DeviceState> g_dev;

DeviceState* device_state(std::string* err) {
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess) {
    set_err(err, "cudaGetDevice failed");
    return nullptr;
  }
  std::lock_guard<std::mutex> lk(g_mu);
  if (static_cast<int>(g_dev.size()) <= dev) g_dev.resize(dev + 1);
  DeviceState& d = g_dev[dev];
  if (!d.init) {
    cudaDeviceProp prop;
    if (cudaGetDeviceProperties(&prop, dev) != cudaSuccess) {
      set_err(err, "cudaGetDeviceProperties failed");
      return nullptr;
    }
    d.sms = prop.multiProcessorCount;
    d.cc_major = prop.major;
    d.cc_minor = prop.minor;
    void* sym = nullptr;
    if (cudaGetSymbolAddress(&sym, g_device_error) != cudaSuccess) {
      set_err(err, "cudaGetSymbolAddress(g_device_error) failed");
      return nullptr;
    }
    d.err_word = static_cast<uint32_t*>(sym);
    d.init = true;
  }
  return &d;
}

// Tensor maps of the peer destinations live in device memory (a kernel parameter would not
// hold seven of them). One small array per distinct set of destinations and shape, built on
// first use and kept for the life of the process (at most 1920 bytes each): an array handed to
// a launch is never freed under it, whichever host thread made the call. Callers that keep
// making new destination sets (new buffers every call) hit the cap and get an error.
struct PeerMapsEntry {
  int dev = -1;
  std::vector<const void*> ptrs;
  long rows = 0, cols = 0, pitch = 0;
  int kind = 0;
  CUtensorMap* d_maps = nullptr;
};
std::vector<PeerMapsEntry> g_peer_maps;
constexpr size_t kPeerMapEntries = 4096;

const CUtensorMap* peer_maps(void* const* peers, int n, const void* local, long rows, long cols,
                             long pitch, int kind, std::string* err) {
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess) {
    set_err(err, "cudaGetDevice failed");
    return nullptr;
  }
  std::vector<const void*> key(peers, peers + n);
  key.push_back(local);
  std::lock_guard<std::mutex> lk(g_mu);
  for (const PeerMapsEntry& e : g_peer_maps)
    if (e.dev == dev && e.ptrs == key && e.rows == rows && e.cols == cols && e.pitch == pitch &&
        e.kind == kind)
      return e.d_maps;
  // FP32: n narrow maps. BF16: n narrow, n wide, then the wide map of the local C.
  const int count = kind == 1 ? 2 * n + 1 : n;
  std::vector<CUtensorMap> maps(count);
  for (int i = 0; i < count; ++i) {
    void* base = const_cast<void*>(i < 2 * n ? static_cast<const void*>(peers[i % n]) : local);
    if (!encode_output_map(&maps[i], base, static_cast<int>(rows), static_cast<int>(cols), pitch,
                           kind == 1, err, i >= n))
      return nullptr;
  }
  if (g_peer_maps.size() >= kPeerMapEntries) {
    set_err(err, "too many distinct peer destination sets (keep the peer buffers and reuse them)");
    return nullptr;
  }
  PeerMapsEntry ne;
  ne.dev = dev;
  ne.ptrs = key;
  ne.rows = rows;
  ne.cols = cols;
  ne.pitch = pitch;
  ne.kind = kind;
  if (cudaMalloc(&ne.d_maps, sizeof(CUtensorMap) * count) != cudaSuccess ||
      cudaMemcpy(ne.d_maps, maps.data(), sizeof(CUtensorMap) * count, cudaMemcpyHostToDevice) !=
          cudaSuccess) {
    if (ne.d_maps) cudaFree(ne.d_maps);
    set_err(err, "cudaMalloc/cudaMemcpy of the peer tensor maps failed");
    return nullptr;
  }
  g_peer_maps.push_back(ne);
  return ne.d_maps;
}

// Output side of a launch: row pitch, the TMA-store decision, the C tensor map and the peer
// destinations. Peers need the TMA-store path (FP32/BF16, 16-byte aligned rows).
bool setup_output(const Nvfp4DeviceOperands& op, GemmParams& p, void* out, CUtensorMap* tc,
                  std::string* err) {
  std::memset(tc, 0, sizeof(*tc));
  p.peer_maps = nullptr;
  p.n_peers = 0;
  const long ldc = op.ldd ? op.ldd : op.N;
  if (ldc < op.N) {
    set_err(err, "ldc must be at least N");
    return false;
  }
  if (p.out_nvfp4 && ldc != op.N) {
    set_err(err, "NVFP4 output takes no ldc");
    return false;
  }
  p.ldc = static_cast<int>(ldc);
  const int esize = p.out_bf16 ? 2 : 4;
  p.tma_store = (!p.out_nvfp4 && (static_cast<size_t>(ldc) * esize) % 16 == 0 &&
                 (reinterpret_cast<uintptr_t>(out) & 15) == 0)
                    ? 1 : 0;
  if (op.n_peers != 0) {
    if (op.n_peers < 0 || op.n_peers > 7 || !op.d_peers) {
      set_err(err, "n_peers must be 0..7 with a c_peers array");
      return false;
    }
    bool aligned = true;
    for (int i = 0; i < op.n_peers; ++i)
      aligned = aligned && op.d_peers[i] && (reinterpret_cast<uintptr_t>(op.d_peers[i]) & 15) == 0;
    if (!p.tma_store || !aligned) {
      set_err(err, "peer outputs need FP32/BF16 output, 16-byte aligned c and c_peers, and "
                   "ldc * element size a multiple of 16");
      return false;
    }
  }
  const int kind = p.out_bf16 ? 1 : 2;
  if (p.tma_store && !cached_map(MapKey{out, op.M, op.N, 32, kind, ldc}, tc, err)) return false;
  if (op.n_peers > 0) {
    p.peer_maps = peer_maps(op.d_peers, op.n_peers, out, op.M, op.N, ldc, kind, err);
    if (!p.peer_maps) return false;
    p.n_peers = op.n_peers;
  }
  return true;
}

template <int BN, bool SP, bool PEERS>
bool launch_dense_as(const CUtensorMap& ta, const CUtensorMap& tb, const CUtensorMap& tc,
                     const GemmParams& p, DeviceState* ds, cudaStream_t s, std::string* err) {
  using C = Cfg<BN, SP>;
  const int idx = (SP ? 2 : (BN == 256 ? 1 : 0)) + (PEERS ? 3 : 0);
  if (!ds->attr_set[idx]) {
    cudaError_t e = cudaFuncSetAttribute(gemm_mxf4nvf4_kernel<BN, SP, PEERS>,
                                         cudaFuncAttributeMaxDynamicSharedMemorySize,
                                         C::kSmemBytes);
    if (e != cudaSuccess) {
      set_err(err, std::string("cudaFuncSetAttribute: ") + cudaGetErrorString(e));
      return false;
    }
    ds->attr_set[idx] = true;
  }
  int grid = p.num_tiles < ds->sms ? p.num_tiles : ds->sms;
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(grid, 1, 1);
  cfg.blockDim = dim3(kNumThreads, 1, 1);
  cfg.dynamicSmemBytes = C::kSmemBytes;
  cfg.stream = s;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  cudaError_t e = cudaLaunchKernelEx(&cfg, gemm_mxf4nvf4_kernel<BN, SP, PEERS>, ta, tb, tc, p);
  if (e == cudaSuccess) e = cudaGetLastError();
  if (e != cudaSuccess) {
    set_err(err, std::string("gemm launch: ") + cudaGetErrorString(e));
    return false;
  }
  return true;
}

// The kernel with the peer stores compiled in only when the call has peer destinations.
template <int BN, bool SP = false>
bool launch_dense(const CUtensorMap& ta, const CUtensorMap& tb, const CUtensorMap& tc,
                  const GemmParams& p, DeviceState* ds, cudaStream_t s, std::string* err) {
  return p.n_peers > 0 ? launch_dense_as<BN, SP, true>(ta, tb, tc, p, ds, s, err)
                       : launch_dense_as<BN, SP, false>(ta, tb, tc, p, ds, s, err);
}

bool launch_pair(const CUtensorMap& ta, const CUtensorMap& tb, const CUtensorMap& tc,
                 const GemmParams& p, DeviceState* ds, cudaStream_t s, std::string* err) {
  using C = PairCfg;
  cudaLaunchConfig_t cfg = {};
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeClusterDimension;
  attr[0].val.clusterDim.x = 2;
  attr[0].val.clusterDim.y = 1;
  attr[0].val.clusterDim.z = 1;
  cfg.blockDim = dim3(kNumThreads, 1, 1);
  cfg.dynamicSmemBytes = C::kSmemBytes;
  cfg.stream = s;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  if (!ds->pair_attr_set) {
    cudaError_t e = cudaFuncSetAttribute(gemm_mxf4nvf4_pair_kernel,
                                         cudaFuncAttributeMaxDynamicSharedMemorySize, C::kSmemBytes);
    if (e != cudaSuccess) {
      set_err(err, std::string("cudaFuncSetAttribute (pair): ") + cudaGetErrorString(e));
      return false;
    }
    int ncl = 0;
    cfg.gridDim = dim3(2 * (ds->sms / 2), 1, 1);
    e = cudaOccupancyMaxActiveClusters(&ncl, gemm_mxf4nvf4_pair_kernel, &cfg);
    if (e != cudaSuccess || ncl < 1) ncl = ds->sms / 2;
    ds->pair_clusters = ncl;
    ds->pair_attr_set = true;
  }
  const int ncl = p.num_tiles < ds->pair_clusters ? p.num_tiles : ds->pair_clusters;
  cfg.gridDim = dim3(2 * ncl, 1, 1);
  cudaError_t e = cudaLaunchKernelEx(&cfg, gemm_mxf4nvf4_pair_kernel, ta, tb, tc, p);
  if (e != cudaSuccess) {
    set_err(err, std::string("gemm (pair) launch: ") + cudaGetErrorString(e));
    return false;
  }
  return true;
}

}  // namespace

size_t sf_tcgen05_bytes(int rows, int K) {
  return static_cast<size_t>((rows + 127) / 128) * static_cast<size_t>((K + 63) / 64) * 512;
}

uint32_t* device_error_word(std::string* err) {
  DeviceState* ds = device_state(err);
  return ds ? ds->err_word : nullptr;
}

// The scale workspace of stream `s` on this device, at least `bytes` long. Growing it frees
// the old buffer (cudaFree waits for the device, so earlier work on the stream has finished).
uint8_t* scale_workspace(DeviceState* ds, cudaStream_t s, size_t bytes, std::string* err) {
  std::lock_guard<std::mutex> lk(g_mu);
  DeviceState::Workspace* w = nullptr;
  for (auto& x : ds->ws)
    if (x.stream == s) w = &x;
  if (!w) {
    ds->ws.push_back(DeviceState::Workspace{s, nullptr, 0});
    w = &ds->ws.back();
  }
  if (w->bytes < bytes) {
    if (w->ptr) cudaFree(w->ptr);
    w->ptr = nullptr;
    w->bytes = 0;
    if (cudaMalloc(&w->ptr, bytes) != cudaSuccess) {
      set_err(err, "cudaMalloc of the scale workspace failed");
      return nullptr;
    }
    w->bytes = bytes;
  }
  return w->ptr;
}

bool gemm_dense(const Nvfp4DeviceOperands& op, cudaStream_t s, std::string* err) {
  DeviceState* ds = device_state(err);
  if (!ds) return false;
  if (ds->cc_major != 10) {
    set_err(err, "the b200 backend needs an sm_100 device (found sm_" +
                     std::to_string(ds->cc_major) + std::to_string(ds->cc_minor) + ")");
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
  if (op.d == nullptr && op.out_dtype != OutDType::F32) {
    set_err(err, "out_dtype BF16 needs the output in `d`");
    return false;
  }
  if (op.M <= 0 || op.N <= 0 || op.K <= 0) {
    set_err(err, "M, N and K must be positive");
    return false;
  }
  if (op.K % 32 != 0) {
    set_err(err, "K must be a multiple of 32 (packed rows must be 16-byte aligned for TMA)");
    return false;
  }
  if ((reinterpret_cast<uintptr_t>(op.a_packed) | reinterpret_cast<uintptr_t>(op.b_packed)) & 15) {
    set_err(err, "packed operands must be 16-byte aligned");
    return false;
  }
  const uint8_t* sfa = op.a_scales;
  const uint8_t* sfb = op.b_scales;
  if (op.sf_layout == SfLayout::Canonical) {
    const size_t na = sf_tcgen05_bytes(op.M, op.K), nb = sf_tcgen05_bytes(op.N, op.K);
    uint8_t* ws = scale_workspace(ds, s, na + nb, err);
    if (!ws) return false;
    if (!sf_to_tcgen05_pair(op.a_scales, op.M, op.b_scales, op.N, op.K, ws, ws + na, s, err)) return false;
    sfa = ws;
    sfb = ws + na;
    // The weight scales the kernel reads were written by the reorder just enqueued, so the
    // caller's B_STATIC promise does not cover them: the GEMM waits for that work in full.
    Nvfp4DeviceOperands o = op;
    o.b_static = false;
    if ((reinterpret_cast<uintptr_t>(sfa) | reinterpret_cast<uintptr_t>(sfb)) & 15) {
      set_err(err, "tcgen05-layout scales must be 16-byte aligned");
      return false;
    }
    return gemm_dense_tc(o, sfa, sfb, out, s, err);
  }
  if ((reinterpret_cast<uintptr_t>(sfa) | reinterpret_cast<uintptr_t>(sfb)) & 15) {
    set_err(err, "tcgen05-layout scales must be 16-byte aligned");
    return false;
  }
  return gemm_dense_tc(op, sfa, sfb, out, s, err);
}

// NVFP4 output parameters (and the zeroed padding of a tcgen05-layout scale buffer); also
// turns the TMA-store path off, which writes FP32/BF16 tiles only.
bool setup_nvfp4_out(const Nvfp4DeviceOperands& op, GemmParams& p, cudaStream_t s, std::string* err) {
  p.out_nvfp4 = op.out_dtype == OutDType::NVFP4 ? 1 : 0;
  p.out_sf = op.d_scales;
  p.out_g = op.d_global;
  p.out_sf_tc = op.d_sf_layout == SfLayout::Tcgen05 ? 1 : 0;
  p.out_ka = (op.N + 63) / 64;
  if (!p.out_nvfp4) return true;
  if (!op.d || !op.d_scales || op.N % 32 != 0 || (reinterpret_cast<uintptr_t>(op.d) & 15) ||
      (reinterpret_cast<uintptr_t>(op.d_scales) & 1)) {
    set_err(err, "NVFP4 output needs d (16-byte aligned) and d_scales, and N a multiple of 32");
    return false;
  }
  if (p.out_sf_tc && op.M % 128 != 0 &&
      cudaMemsetAsync(op.d_scales, 0, sf_tcgen05_bytes(op.M, op.N), s) != cudaSuccess) {
    set_err(err, "cudaMemsetAsync of the output scale buffer failed");
    return false;
  }
  return true;
}

bool gemm_dense_tc(const Nvfp4DeviceOperands& op, const uint8_t* sfa, const uint8_t* sfb,
                   void* out, cudaStream_t s, std::string* err) {
  DeviceState* ds = device_state(err);
  if (!ds) return false;
  // At most one 128-row block of tokens (decode): the weight-streaming kernel (weight rows on
  // the MMA's 128-row side, one CTA per SM, split-K over a cluster when the weight has fewer
  // 128-row tiles than there are SMs). An explicit tile shape or SM grouping selects the
  // general kernel.
  if (op.M <= 128 && op.cta_group == 0 && op.tile_n == 0 && op.out_dtype != OutDType::NVFP4 &&
      (op.ldd == 0 || op.ldd == op.N) && op.n_peers == 0)
    return gemm_decode(op, sfa, sfb, out, s, err);
  int bn = op.tile_n;
  const int tiles_m = (op.M + kBM - 1) / kBM;
  // Default: one-SM tiles (measured faster than the SM-pair kernel on B200 so far); the
  // SM-pair kernel (256 x 256 tiles) on request.
  int cg = op.cta_group;
  if (cg == 0) cg = 1;
  if (cg != 1 && cg != 2) {
    set_err(err, "cta_group must be 0, 1 or 2");
    return false;
  }
  if (cg == 2) {
    if (bn != 0 && bn != 256) {
      set_err(err, "SM-pair tiles are 256 x 256 (tile_n must be 0 or 256 with cta_group 2)");
      return false;
    }
    bn = 256;
  }
  if (bn == 0) bn = (static_cast<long>(tiles_m) * ((op.N + 255) / 256) >= ds->sms) ? 256 : 128;
  if (bn != 128 && bn != 256) {
    set_err(err, "tile_n must be 128 or 256 for the dense kernel");
    return false;
  }
  GemmParams p;
  p.sfa = sfa;
  p.sfb = sfb;
  p.meta = nullptr;
  p.out = out;
  p.M = op.M;
  p.N = op.N;
  p.K = op.K;
  p.ldc = op.N;
  p.alpha = op.a_global * op.b_global;
  p.out_bf16 = (op.d != nullptr && op.out_dtype == OutDType::BF16) ? 1 : 0;
  p.tiles_m = cg == 2 ? (op.M + 255) / 256 : tiles_m;
  p.tiles_n = (op.N + bn - 1) / bn;
  p.num_tiles = p.tiles_m * p.tiles_n;
  p.ka = (op.K + 63) / 64;
  p.num_kt = (op.K + 255) / 256;
  p.sfb_rowblocks = (op.N + 127) / 128;
  p.sfa_rowblocks = (op.M + 127) / 128;
  // Tile raster: groups of group_m tile rows walked down M first, so one band of B is reused by
  // a whole group while it is in L2 (32 one-SM rows: 1% faster than 16 at C2 and C4, 8 slower).
  p.group_m = cg == 2 ? 8 : 32;
  p.err_word = ds->err_word;
  if (!setup_nvfp4_out(op, p, s, err)) return false;
  CUtensorMap ta, tb;
  if (!cached_map(MapKey{op.a_packed, op.M, op.K, kBM, 0}, &ta, err)) return false;
  if (!cached_map(MapKey{op.b_packed, op.N, op.K, cg == 2 ? 128 : bn, 0}, &tb, err)) return false;
  CUtensorMap tc;
  if (!setup_output(op, p, out, &tc, err)) return false;
  if (cg == 2) return launch_pair(ta, tb, tc, p, ds, s, err);
  return bn == 256 ? launch_dense<256>(ta, tb, tc, p, ds, s, err)
                   : launch_dense<128>(ta, tb, tc, p, ds, s, err);
}

// GemmMode::Sparse: A compressed ([M][K/4] kept pair bytes) + metadata ([M][K/16]) + block-32
// scales; B dense with block-32 scales (see the sparse kernel's comment).
bool gemm_sparse(const Nvfp4DeviceOperands& op, cudaStream_t s, std::string* err) {
  DeviceState* ds = device_state(err);
  if (!ds) return false;
  if (ds->cc_major != 10) {
    set_err(err, "the b200 backend needs an sm_100 device");
    return false;
  }
  if (!op.a_packed || !op.b_packed || !op.a_scales || !op.b_scales || !op.a_meta) {
    set_err(err, "sparse mode needs compressed A, its metadata (a_meta), B and both scales");
    return false;
  }
  void* out = op.d ? op.d : static_cast<void*>(op.c);
  if (!out) {
    set_err(err, "null output pointer");
    return false;
  }
  if (op.d == nullptr && op.out_dtype != OutDType::F32) {
    set_err(err, "out_dtype BF16 needs the output in `d`");
    return false;
  }
  if (op.M <= 0 || op.N <= 0 || op.K <= 0 || op.K % 128 != 0) {
    set_err(err, "sparse mode needs positive M, N and K a multiple of 128");
    return false;
  }
  if (op.cta_group == 2 || (op.tile_n != 0 && op.tile_n != 256)) {
    set_err(err, "sparse mode runs 128 x 256 one-SM tiles (cta_group 0/1, tile_n 0/256)");
    return false;
  }
  if ((reinterpret_cast<uintptr_t>(op.a_packed) | reinterpret_cast<uintptr_t>(op.b_packed)) & 15 ||
      (reinterpret_cast<uintptr_t>(op.a_meta) & 3)) {
    set_err(err, "packed operands must be 16-byte aligned and the metadata 4-byte aligned");
    return false;
  }
  // Block-32 scales: the tcgen05 layout of a block-16 operand of K/2 columns.
  const int vk = op.K / 2;
  const uint8_t* sfa = op.a_scales;
  const uint8_t* sfb = op.b_scales;
  if (op.sf_layout == SfLayout::Canonical) {
    const size_t na = sf_tcgen05_bytes(op.M, vk), nb = sf_tcgen05_bytes(op.N, vk);
    uint8_t* ws = scale_workspace(ds, s, na + nb, err);
    if (!ws) return false;
    if (!sf_to_tcgen05_pair(op.a_scales, op.M, op.b_scales, op.N, vk, ws, ws + na, s, err)) return false;
    sfa = ws;
    sfb = ws + na;
  }
  if ((reinterpret_cast<uintptr_t>(sfa) | reinterpret_cast<uintptr_t>(sfb)) & 15) {
    set_err(err, "tcgen05-layout scales must be 16-byte aligned");
    return false;
  }
  GemmParams p;
  p.sfa = sfa;
  p.sfb = sfb;
  p.meta = op.a_meta;
  p.out = out;
  p.M = op.M;
  p.N = op.N;
  p.K = op.K;
  p.ldc = op.N;
  p.alpha = op.a_global * op.b_global;
  p.out_bf16 = (op.d != nullptr && op.out_dtype == OutDType::BF16) ? 1 : 0;
  p.tiles_m = (op.M + 127) / 128;
  p.tiles_n = (op.N + 255) / 256;
  p.num_tiles = p.tiles_m * p.tiles_n;
  p.group_m = 32;
  p.ka = (op.K + 127) / 128;          // MMAs (and scale atoms) along K
  p.num_kt = (op.K + 255) / 256;      // 256-K stages
  p.sfb_rowblocks = (op.N + 127) / 128;
  p.sfa_rowblocks = (op.M + 127) / 128;
  p.err_word = ds->err_word;
  if (!setup_nvfp4_out(op, p, s, err)) return false;
  CUtensorMap ta, tb, tc;
  // Compressed A: [M][K/4] bytes, i.e. a packed operand of K/2 columns, in 64-byte boxes.
  if (!cached_map(MapKey{op.a_packed, op.M, vk, 128, 3}, &ta, err)) return false;
  if (!cached_map(MapKey{op.b_packed, op.N, op.K, 256, 0}, &tb, err)) return false;
  if (!setup_output(op, p, out, &tc, err)) return false;
  return launch_dense<256, true>(ta, tb, tc, p, ds, s, err);
}

bool operand_map(CUtensorMap* map, const void* base, int rows, int K, int box_rows,
                 std::string* err) {
  return cached_map(MapKey{base, rows, K, box_rows, 0}, map, err);
}

int device_sms(std::string* err) {
  DeviceState* ds = device_state(err);
  return ds ? ds->sms : 0;
}

int device_cc_major(std::string* err) {
  DeviceState* ds = device_state(err);
  return ds ? ds->cc_major : 0;
}

bool wait_selftest(uint64_t limit_ns, std::string* err) {
  DeviceState* ds = device_state(err);
  if (!ds) return false;
  wait_selftest_kernel<<<1, 32>>>(limit_ns, ds->err_word);
  cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) {
    set_err(err, std::string("selftest launch: ") + cudaGetErrorString(e));
    return false;
  }
  return true;
}

}  // namespace nvfp4b200

// src/gemm.h:27-29 signature; registered in launch_gemm (include/gemm.h).
bool launch_gemm_b200(const Nvfp4DeviceOperands& op, cudaStream_t s, std::string* err) {
  if (op.mode == GemmMode::Sparse) return nvfp4b200::gemm_sparse(op, s, err);
  return nvfp4b200::gemm_dense(op, s, err);
}
