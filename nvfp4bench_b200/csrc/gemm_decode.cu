// gemm_decode.cu - weight-streaming NVFP4 GEMM for decode shapes (M <= 128 tokens).
//
// The decode configurations (M in {16, 64, 128} tokens x a 14336 x 4096 or 4096 x 14336
// weight) are HBM-bound: the weight B is read once and everything else is small. The general
// kernel tiles M by 128 rows, so at M = 16 it keeps at most N/256 CTAs busy and runs the MMA
// at 1/8 of its M; this kernel turns the problem around:
//   * the weight rows are the MMA's 128-row "A" side (D^T = B * A^T in TMEM, lane = weight
//     row n), the tokens its "B" side with N = M rounded up to 16..128;
//   * one CTA per SM, each streaming its share of the weight through a deep ring of shared
//     memory stages (6 to 10, about 190 KB in flight per SM);
//   * when there are fewer 128-row weight tiles than SMs, the K range of a tile is split over
//     the S CTAs of one thread-block cluster (S = 2, 4 or 8). Each CTA parks its FP32 partial
//     sums in its own shared memory, and after a cluster barrier CTA r adds up its share of
//     the tokens from all S partials through distributed shared memory, in rank order
//     (deterministic), and stores C. No workspace, no atomics, no second pass.
// The epilogue needs no transpose: thread = weight row n holds the values of all tokens, so a
// warp stores 32 consecutive columns of C per token.
//
// Roles (320 threads): warp 0 producer (per stage: the weight and token tiles by TMA onto
// "full", the stage's weight and token scale atoms by bulk copy onto "sfd"), warp 1 MMA
// issuer, warps 2..5 epilogue, warps 6..9 scale writers. The writers move each stage's scales
// from shared memory into a ring of three TMEM scale slots: weight scales (the MMA's A side,
// rows = TMEM lanes) one column per quadrant, the one its MMA rows read; token scales (B
// side) whole in every quadrant. (Loading them from global memory in the writers themselves
// put an L2 round trip per stage on the critical path: one writer group, one stage at a
// time.) Bounded waits as everywhere (ptx.cuh).
#include <cuda.h>
#include <cuda_bf16.h>
#include <cuda_runtime.h>

#include <mutex>
#include <string>
#include <vector>

#include "gemm.h"
#include "codec_dev.cuh"
#include "internal.h"
#include "ptx.cuh"

namespace nvfp4b200 {
namespace {

constexpr int kDThreads = 320;
constexpr int kDTmemCols = 512;   // accumulator [0, 128) + kDSfSlots slots of 32 columns
constexpr int kDSfSlots = 12;     // at most; deep enough that the slot ring never throttles
constexpr int kDMaxCluster = 8;
constexpr int kDSmemBudget = 220 * 1024;

// Grid barrier of the fused quantisation: every CTA's quantiser warps add 1 to `arrive` when
// their slice of A is written; each producer waits for `arrive` to reach the grid size and
// then adds 1 to `depart`; the last to depart resets both, so each launch starts from zero.
// (The next launch on the stream reads them only after this grid has completed.)
__device__ unsigned int g_qa_arrive = 0;
__device__ unsigned int g_qa_depart = 0;

__device__ __forceinline__ unsigned int ld_acquire_gpu(const unsigned int* p) {
  unsigned int v;
  asm volatile("ld.acquire.gpu.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
  return v;
}
__device__ __forceinline__ void fence_proxy_async_global() {
  asm volatile("fence.proxy.async.global;" ::: "memory");
}

struct DParams {
  const uint8_t* sfw;   // weight (MMA A side) scales, tcgen05 layout over N rows
  const uint8_t* sft;   // token (MMA B side) scales, tcgen05 layout over M rows
  void* out;
  int M, N, K;
  float alpha;
  int out_bf16;
  int tiles_n, splits, num_kt, ka;
  int b_static;         // the weight may be read before the preceding kernel completes
  int vec_out;          // C rows and pointer allow 16-byte stores (N * element size % 16 == 0)
  // Fused activation quantisation (a_src != null): the CTAs first quantise fp32 A [M][K] into
  // the token operand (packed `a_packed` [M][K/2], tcgen05 scales `sft`) with global scale
  // a_g, exactly as the standalone quantiser does, then meet at a grid barrier before any
  // token tile is loaded. The weight stream does not wait for it.
  const float* a_src;
  uint8_t* a_packed;
  float a_g;
  uint32_t* err_word;
};

// A stage is KB = 8 K-blocks of 64 (K = 512, two 128-byte-wide TMA boxes per operand; at
// least three stages fit for every token count). Per-stage costs (barrier waits, two commits,
// fences: about 370 cycles measured beside the MMAs' own 4 x 46 cycles at N = 16) then fall
// on twice the weight bytes; a 16 KB stage every ~620 cycles is what one SM's share of HBM
// bandwidth delivers.
template <int MPAD>
struct DCfg {
  static constexpr int kKb = 8;                       // K-blocks per stage
  static constexpr int kHalves = kKb / 4;             // 128-byte-wide boxes per operand
  static constexpr int kWBytes = kHalves * 128 * 128; // 128 weight rows x 256 FP4 per box
  static constexpr int kTBytes = kHalves * MPAD * 128;
  static constexpr int kSfBytes = kKb * 512;          // one 128-row atom per K-block
  static constexpr int kStageBytes = kWBytes + kTBytes + 2 * kSfBytes;
  static constexpr int kStages0 = kDSmemBudget / kStageBytes;
  static constexpr int kStages = kStages0 > 10 ? 10 : kStages0;
  // TMEM scale slot: weight scales at +4*kb (column 4*kb + q used by quadrant q), token
  // scales at +4*kKb + 4*kb.
  static constexpr int kSlotCols = 8 * kKb;
  static constexpr int kSlots0 = (kDTmemCols - 128) / kSlotCols;
  static constexpr int kSlots1 = kSlots0 < kDSfSlots ? kSlots0 : kDSfSlots;
  // A writer's slot wait (the MMA of stage i - slots finished) must also order its "full"
  // arrival after that barrier's previous phase (stage i - stages): slots <= stages.
  static constexpr int kSlots = kSlots1 < kStages ? kSlots1 : kStages;
  static constexpr int kPartBytes = MPAD * 128 * 4;   // FP32 partial sums, [token][row]
  static constexpr int kSmemBytes = 1024 + kStages * kStageBytes + 512;
  static_assert(kPartBytes <= kStages * kStageBytes, "partials reuse the stage memory");
  static_assert(kStages >= 3, "pipeline depth");
  static_assert(kSmemBytes <= 232448, "shared memory budget");
};

__device__ __forceinline__ void store_out(const DParams& p, int m, int n, float v) {
  if (p.out_bf16)
    reinterpret_cast<__nv_bfloat16*>(p.out)[static_cast<size_t>(m) * p.N + n] = __float2bfloat16_rn(v);
  else
    reinterpret_cast<float*>(p.out)[static_cast<size_t>(m) * p.N + n] = v;
}

__device__ __forceinline__ float4 ld_dsmem_f32x4(uint32_t cluster_addr) {
  float4 v;
  asm volatile("ld.shared::cluster.v4.f32 {%0, %1, %2, %3}, [%4];"
               : "=f"(v.x), "=f"(v.y), "=f"(v.z), "=f"(v.w)
               : "r"(cluster_addr)
               : "memory");
  return v;
}

template <int MPAD>
__global__ void __launch_bounds__(kDThreads, 1)
    gemm_decode_kernel(const __grid_constant__ CUtensorMap tmap_w,
                       const __grid_constant__ CUtensorMap tmap_t, const DParams p) {
  using C = DCfg<MPAD>;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) &
                                             ~uintptr_t(1023));
  uint8_t* sW = smem;
  uint8_t* sT = sW + C::kStages * C::kWBytes;
  uint8_t* sSFW = sT + C::kStages * C::kTBytes;
  uint8_t* sSFT = sSFW + C::kStages * C::kSfBytes;
  float* part = reinterpret_cast<float*>(smem);  // after the last MMA: [MPAD][128] partials
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + C::kStages * C::kStageBytes);
  uint64_t* full = bars;                      // operand bytes + producer + 4 scale writers
  uint64_t* empty = full + C::kStages;        // smem stage consumed
  uint64_t* sfd = empty + C::kStages;         // the stage's scale atoms landed
  uint64_t* acc_full = sfd + C::kStages;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(acc_full + 1);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  // Cluster = the K splits of one weight tile (cluster dims (splits, 1, 1)).
  const int ks = static_cast<int>(blockIdx.x) % p.splits;
  const int tn = static_cast<int>(blockIdx.x) / p.splits;
  const int kt0 = static_cast<int>(static_cast<long>(ks) * p.num_kt / p.splits);
  const int kt1 = static_cast<int>(static_cast<long>(ks + 1) * p.num_kt / p.splits);

  if (threadIdx.x == 0) {
    for (int s = 0; s < C::kStages; ++s) {
      mbar_init(smem_u32(&full[s]), 1 + 4);
      mbar_init(smem_u32(&empty[s]), 1);
      mbar_init(smem_u32(&sfd[s]), 1);
    }
    mbar_init(smem_u32(acc_full), 1);
    *abort_flag = 0;
    fence_mbar_init();
    prefetch_tmap(&tmap_w);
    prefetch_tmap(&tmap_t);
  }
  if (warp == 1) {
    tmem_alloc(smem_u32(tmem_slot), kDTmemCols);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem_base = *tmem_slot;
  // Launched with programmatic stream serialization: the set-up above overlaps the previous
  // kernel on the stream. Every thread that reads or writes global memory first waits for
  // that kernel to complete (griddepcontrol.wait) - except that with b_static the producer
  // starts loading the first stages' weight bytes before its wait (the caller guarantees the
  // weight is not written by the preceding work), so the weight stream overlaps e.g. the
  // quantisation of this layer's activations.
  asm volatile("griddepcontrol.launch_dependents;" ::: "memory");

  if (p.a_src && warp >= 2) {
    // ------------------------------------------------- fused activation quantisation (phase 1)
    // Warps 2..9 (idle until the first stage) quantise this CTA's share of the 16-element
    // blocks of A (src/nvfp4.cu:62-97 through the codec's device code) and write the packed
    // values and tcgen05-layout scales; scale bytes of the padding rows up to 128 are zeroed,
    // as the standalone quantiser leaves them.
    asm volatile("griddepcontrol.wait;" ::: "memory");  // A is the previous kernel's output
    const int nb = p.K / 16;
    const long rows_pad = (static_cast<long>(p.M) + 127) / 128 * 128;
    const long total = rows_pad * nb;
    const long per = (total + gridDim.x - 1) / gridDim.x;
    const long b0 = per * blockIdx.x;
    const long b1 = b0 + per < total ? b0 + per : total;
    for (long b = b0 + (threadIdx.x - 64); b < b1; b += kDThreads - 64) {
      const int r = static_cast<int>(b / nb), c = static_cast<int>(b % nb);
      uint8_t sc = 0;
      if (r < p.M) {
        const float4* x4 = reinterpret_cast<const float4*>(p.a_src + static_cast<size_t>(r) * p.K + c * 16);
        float x[16];
#pragma unroll
        for (int v = 0; v < 4; ++v) {
          const float4 t = x4[v];
          x[4 * v] = t.x; x[4 * v + 1] = t.y; x[4 * v + 2] = t.z; x[4 * v + 3] = t.w;
        }
        uint32_t lo, hi;
        sc = quantize16_dev(x, p.a_g, lo, hi);
        *reinterpret_cast<uint2*>(p.a_packed + (static_cast<size_t>(r) * p.K + c * 16) / 2) = make_uint2(lo, hi);
      }
      const size_t atom = static_cast<size_t>(r / 128) * p.ka + c / 4;
      const_cast<uint8_t*>(p.sft)[atom * 512 + (r % 32) * 16 + ((r / 32) % 4) * 4 + (c % 4)] = sc;
    }
    fence_proxy_async_global();  // the token tiles are read back by TMA (async proxy)
    __threadfence();
    asm volatile("bar.sync 2, 256;" ::: "memory");
    if (threadIdx.x == 64) atomicAdd(&g_qa_arrive, 1u);
  }

  if (warp == 0) {
    // ---------------------------------------------------------------- TMA producer
    if (lane == 0) {
      bool ok = true;
      int i = 0;
      // Weight half of a stage (tiles + scale atoms) and token half; both count their bytes
      // on the stage's barriers, which expect the whole stage up front.
      auto issue_w = [&](int kt, int s) {
        int nkb = p.ka - kt * C::kKb;
        if (nkb > C::kKb) nkb = C::kKb;
        const uint32_t sfb = static_cast<uint32_t>(nkb) * 512u;
        const uint32_t db = smem_u32(&sfd[s]), fb = smem_u32(&full[s]);
        mbar_arrive_expect_tx(db, 2 * sfb);
        mbar_arrive_expect_tx(fb, C::kWBytes + C::kTBytes);
        bulk_load(smem_u32(sSFW + s * C::kSfBytes),
                  p.sfw + (static_cast<size_t>(tn) * p.ka + kt * C::kKb) * 512, sfb, db);
        // Boxes past the end of K read as zeros (and still count their bytes).
#pragma unroll
        for (int h = 0; h < C::kHalves; ++h)
          tma_load_2d(smem_u32(sW + s * C::kWBytes + h * 128 * 128), &tmap_w,
                      kt * C::kKb * 32 + h * 128, tn * 128, fb);
      };
      auto issue_t = [&](int kt, int s) {
        int nkb = p.ka - kt * C::kKb;
        if (nkb > C::kKb) nkb = C::kKb;
        bulk_load(smem_u32(sSFT + s * C::kSfBytes), p.sft + static_cast<size_t>(kt) * C::kKb * 512,
                  static_cast<uint32_t>(nkb) * 512u, smem_u32(&sfd[s]));
#pragma unroll
        for (int h = 0; h < C::kHalves; ++h)
          tma_load_2d(smem_u32(sT + s * C::kTBytes + h * MPAD * 128), &tmap_t,
                      kt * C::kKb * 32 + h * 128, 0, smem_u32(&full[s]));
      };
      // The first pass through the ring needs no "empty" wait.
      int pre = 0;
      if (p.b_static) {
        pre = kt1 - kt0 < C::kStages ? kt1 - kt0 : C::kStages;
        for (int q2 = 0; q2 < pre; ++q2) issue_w(kt0 + q2, q2);
      }
      asm volatile("griddepcontrol.wait;" ::: "memory");
      if (p.a_src) {
        // Phase 2 of the fused quantisation: every CTA's slice of A is written.
        const uint64_t t0 = globaltimer_ns();
        while (ld_acquire_gpu(&g_qa_arrive) < gridDim.x) {
          __nanosleep(64);
          if (globaltimer_ns() - t0 > kWaitLimitNs) {
            *abort_flag = 1;
            atomicOr(p.err_word, kErrWaitTmaFull);
            ok = false;
            break;
          }
        }
        fence_proxy_async_global();
        if (atomicAdd(&g_qa_depart, 1u) == gridDim.x - 1) {
          atomicExch(&g_qa_arrive, 0u);
          atomicExch(&g_qa_depart, 0u);
        }
      }
      if (ok)
        for (int q2 = 0; q2 < pre; ++q2) issue_t(kt0 + q2, q2);
      i = pre;
      for (int kt = kt0 + pre; kt < kt1 && ok; ++kt, ++i) {
        const int s = i % C::kStages;
        const uint32_t j = static_cast<uint32_t>(i / C::kStages);
        if (!mbar_wait(smem_u32(&empty[s]), (j & 1u) ^ 1u, abort_flag, p.err_word,
                       kErrWaitSmemEmpty)) {
          ok = false;
          break;
        }
        issue_w(kt, s);
        issue_t(kt, s);
      }
      if (!ok) {
        // The most recent fill of every stage lands before the CTA exits ("full" also counts
        // the writers, which may have left early: the bounded wait then outlasts the copy).
        for (int back = 1; back <= C::kStages && i - back >= 0; ++back) {
          const int f = i - back;
          volatile int never = 0;
          mbar_wait(smem_u32(&sfd[f % C::kStages]), static_cast<uint32_t>(f / C::kStages) & 1u,
                    &never, p.err_word, kErrWaitDrain);
          mbar_wait(smem_u32(&full[f % C::kStages]), static_cast<uint32_t>(f / C::kStages) & 1u,
                    &never, p.err_word, kErrWaitDrain);
        }
      }
    }
  } else if (warp == 1) {
    // ---------------------------------------------------------------- MMA issuer
    if (lane == 0) {
      const uint32_t idesc = make_idesc_mxf4nvf4(128, MPAD);
      bool ok = true, issued = false;
      int i = 0;
      for (int kt = kt0; kt < kt1; ++kt, ++i) {
        const int s = i % C::kStages;
        const int slot = i % C::kSlots;
        const uint32_t j = static_cast<uint32_t>(i / C::kStages);
        if (!mbar_spin_wait<false>(smem_u32(&full[s]), j & 1u, abort_flag, p.err_word,
                                   kErrWaitTmaFull)) {
          ok = false;
          break;
        }
        tc_fence_after();
        int nkb = p.ka - kt * C::kKb;
        if (nkb > C::kKb) nkb = C::kKb;
        const uint32_t sf_t = tmem_base + 128 + slot * C::kSlotCols;
        // K-block kb: box kb / 4, 32-byte step kb % 4 (+2 in 16-byte descriptor units).
        auto mma = [&](int kb) {
          const int h = kb >> 2, kk = kb & 3;
          const uint64_t ad = make_sdesc(smem_u32(sW + s * C::kWBytes + h * 128 * 128), 16, 1024, 2);
          const uint64_t bd = make_sdesc(smem_u32(sT + s * C::kTBytes + h * MPAD * 128), 16, 1024, 2);
          tc_mma_mxf4nvf4(tmem_base, ad + 2 * kk, bd + 2 * kk, idesc, sf_t + kb * 4,
                          sf_t + 4 * C::kKb + kb * 4, (i > 0 || kb > 0) ? 1u : 0u);
        };
        if (nkb == C::kKb) {
#pragma unroll
          for (int kb = 0; kb < C::kKb; ++kb) mma(kb);
        } else {
          for (int kb = 0; kb < nkb; ++kb) mma(kb);
        }
        issued = true;
        tc_commit(smem_u32(&empty[s]));  // also frees the stage's TMEM scale slot
      }
      // acc_full also tells the epilogue that every MMA has finished reading shared memory.
      if (ok || issued) tc_commit(smem_u32(acc_full));
      if (!ok && issued) {
        volatile int never = 0;
        mbar_wait(smem_u32(acc_full), 0, &never, p.err_word, kErrWaitDrain);
      }
    }
  } else if (warp >= 6) {
    // ---------------------------------------------------------------- scale writers
    const int q = warp & 3;
    const uint32_t lane_base = tmem_base + (static_cast<uint32_t>(q * 32) << 16);
    int i = 0;
    for (int kt = kt0; kt < kt1; ++kt, ++i) {
      const int s = i % C::kStages;
      const int slot = i % C::kSlots;
      const uint32_t j = static_cast<uint32_t>(i / C::kStages);
      // One writer group takes every stage in order, so "sfd" is never two phases ahead.
      if (!mbar_wait(smem_u32(&sfd[s]), j & 1u, abort_flag, p.err_word, kErrWaitTmaFull)) break;
      // Weight rows are TMEM lanes: quadrant q's MMA rows read only word q of each atom row.
      // Token rows map to accumulator columns, read by every quadrant: all four words. Atoms
      // past the end of K hold stale bytes that no MMA reads.
      uint32_t vw[C::kKb], vt[4 * C::kKb];
#pragma unroll
      for (int kb = 0; kb < C::kKb; ++kb) {
        vw[kb] = *reinterpret_cast<const uint32_t*>(sSFW + s * C::kSfBytes + kb * 512 + lane * 16 + q * 4);
        const uint4 t = *reinterpret_cast<const uint4*>(sSFT + s * C::kSfBytes + kb * 512 + lane * 16);
        vt[4 * kb] = t.x; vt[4 * kb + 1] = t.y; vt[4 * kb + 2] = t.z; vt[4 * kb + 3] = t.w;
      }
      // The slot's previous use (stage u = i - kSlots) is consumed once phase u / kStages of
      // that stage's "empty" completes; the next phase needs this writer's own stage first.
      if (i >= C::kSlots) {
        const int u = i - C::kSlots;
        if (!mbar_wait(smem_u32(&empty[u % C::kStages]), static_cast<uint32_t>(u / C::kStages) & 1u,
                       abort_flag, p.err_word, kErrWaitSfEmpty))
          break;
      }
      tc_fence_after();
      const uint32_t sf_t = lane_base + 128 + slot * C::kSlotCols;
#pragma unroll
      for (int kb = 0; kb < C::kKb; ++kb) tmem_st_32x32b_x1(sf_t + kb * 4 + q, vw[kb]);
#pragma unroll
      for (int c = 0; c < C::kKb / 4; ++c) tmem_st_32x32b_x16(sf_t + 4 * C::kKb + 16 * c, vt + 16 * c);
      tc_wait_st();
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(smem_u32(&full[s]));
    }
  } else {
    // ---------------------------------------------------------------- epilogue
    // Thread = weight row n (TMEM lane), registers = tokens.
    const int q = warp & 3;
    const int n_local = q * 32 + lane;
    const int n = tn * 128 + n_local;
    const bool ok = mbar_wait(smem_u32(acc_full), 0, abort_flag, p.err_word, kErrWaitAccFull);
    asm volatile("griddepcontrol.wait;" ::: "memory");  // before any store of C
    tc_fence_after();
    const uint32_t acc_t = tmem_base + (static_cast<uint32_t>(q * 32) << 16);
    // Whole weight tiles with 16-byte-storable rows go through shared memory (the stage ring,
    // idle once every MMA has completed): each thread writes its row's values token by token
    // (a warp writes 32 consecutive columns), then the four warps store [token][128 columns]
    // rows with 16-byte vectors. Thread-per-row scalar stores took ~6 us at M = 128.
    const bool staged = p.splits == 1 && p.vec_out && (tn + 1) * 128 <= p.N;
    const int esz = p.out_bf16 ? 2 : 4;
    uint8_t* tile = smem;  // [MPAD][128] elements of the output type
#pragma unroll
    for (int c0 = 0; c0 < MPAD; c0 += 32) {
      uint32_t r[32];
      tmem_ld_32x32b_x32(acc_t + c0, r);
      tc_wait_ld();
      if (p.splits == 1 && staged) {
#pragma unroll
        for (int jj = 0; jj < 32; ++jj) {
          if (c0 + jj >= MPAD) break;
          const float v = __uint_as_float(r[jj]) * p.alpha;
          uint8_t* d = tile + (static_cast<size_t>(c0 + jj) * 128 + n_local) * esz;
          if (p.out_bf16) *reinterpret_cast<__nv_bfloat16*>(d) = __float2bfloat16_rn(v);
          else *reinterpret_cast<float*>(d) = v;
        }
      } else if (p.splits == 1) {
        if (ok && n < p.N) {
#pragma unroll
          for (int jj = 0; jj < 32; ++jj)
            if (c0 + jj < MPAD && c0 + jj < p.M)
              store_out(p, c0 + jj, n, __uint_as_float(r[jj]) * p.alpha);
        }
      } else {
#pragma unroll
        for (int jj = 0; jj < 32; ++jj)
          if (c0 + jj < MPAD) part[(c0 + jj) * 128 + n_local] = __uint_as_float(r[jj]);
      }
    }
    if (staged) {
      asm volatile("bar.sync 1, 128;" ::: "memory");  // the four epilogue warps
      if (ok) {
        const int vpr = 128 * esz / 16;  // 16-byte vectors per token row
        const int tid = threadIdx.x - 64;
        for (int idx = tid; idx < p.M * vpr; idx += 128) {
          const int m = idx / vpr, v = idx - m * vpr;
          const uint4 x = reinterpret_cast<const uint4*>(tile)[idx];
          *reinterpret_cast<uint4*>(static_cast<uint8_t*>(p.out) +
                                    (static_cast<size_t>(m) * p.N + tn * 128) * esz + v * 16) = x;
        }
      }
    }
  }

  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  if (warp == 1) tmem_dealloc(tmem_base, kDTmemCols);

  if (p.splits > 1) {
    asm volatile("griddepcontrol.wait;" ::: "memory");  // before any store of C
    // Every CTA of the cluster has its partials in shared memory after this barrier.
    cluster_sync();
    // CTA ks reduces tokens [m0, m1) over the cluster, in rank order.
    const int per = (MPAD + p.splits - 1) / p.splits;
    const int m0 = ks * per;
    int m1 = m0 + per;
    if (m1 > p.M) m1 = p.M;
    const uint32_t part_s = smem_u32(part);
    uint32_t peer[kDMaxCluster];
#pragma unroll
    for (int r = 0; r < kDMaxCluster; ++r)
      peer[r] = r < p.splits ? mapa_shared(part_s, static_cast<uint32_t>(r)) : 0u;
    if (*abort_flag == 0) {
      // float4 units: 32 per token row of 128 weight rows.
      for (int idx = m0 * 32 + static_cast<int>(threadIdx.x); idx < m1 * 32; idx += kDThreads) {
        float4 v[kDMaxCluster];
#pragma unroll
        for (int r = 0; r < kDMaxCluster; ++r)
          if (r < p.splits) v[r] = ld_dsmem_f32x4(peer[r] + static_cast<uint32_t>(idx) * 16u);
        float4 acc = v[0];
#pragma unroll
        for (int r = 1; r < kDMaxCluster; ++r)
          if (r < p.splits) {
            acc.x += v[r].x; acc.y += v[r].y; acc.z += v[r].z; acc.w += v[r].w;
          }
        const int m = idx >> 5, nn = tn * 128 + (idx & 31) * 4;
        const float o[4] = {acc.x * p.alpha, acc.y * p.alpha, acc.z * p.alpha, acc.w * p.alpha};
        if (p.vec_out && nn + 4 <= p.N) {
          // Four consecutive columns in one 8-byte (BF16) or 16-byte (FP32) store.
          const size_t off = static_cast<size_t>(m) * p.N + nn;
          if (p.out_bf16) {
            __nv_bfloat162 lo = __floats2bfloat162_rn(o[0], o[1]), hi = __floats2bfloat162_rn(o[2], o[3]);
            uint2 w;
            w.x = *reinterpret_cast<uint32_t*>(&lo);
            w.y = *reinterpret_cast<uint32_t*>(&hi);
            *reinterpret_cast<uint2*>(reinterpret_cast<__nv_bfloat16*>(p.out) + off) = w;
          } else {
            *reinterpret_cast<float4*>(reinterpret_cast<float*>(p.out) + off) = make_float4(o[0], o[1], o[2], o[3]);
          }
        } else {
#pragma unroll
          for (int u = 0; u < 4; ++u)
            if (nn + u < p.N) store_out(p, m, nn + u, o[u]);
        }
      }
    }
    // No CTA leaves while a peer may still read its shared memory.
    cluster_sync();
  }
}

struct DecodeState {
  bool attr[4] = {false, false, false, false};
};
std::mutex g_dmu;
std::vector<DecodeState> g_dstate;

template <int MPAD>
bool launch_decode(const CUtensorMap& tw, const CUtensorMap& tt, DParams p, int sms,
                   DecodeState& st, int idx, cudaStream_t s, std::string* err) {
  using C = DCfg<MPAD>;
  p.num_kt = (p.ka + C::kKb - 1) / C::kKb;
  if (!st.attr[idx]) {
    cudaError_t e = cudaFuncSetAttribute(gemm_decode_kernel<MPAD>,
                                         cudaFuncAttributeMaxDynamicSharedMemorySize, C::kSmemBytes);
    if (e == cudaSuccess)
      e = cudaFuncSetAttribute(gemm_decode_kernel<MPAD>,
                               cudaFuncAttributeNonPortableClusterSizeAllowed, 1);
    if (e != cudaSuccess) {
      set_err(err, std::string("cudaFuncSetAttribute (decode): ") + cudaGetErrorString(e));
      return false;
    }
    st.attr[idx] = true;
  }
  cudaLaunchConfig_t cfg = {};
  cudaLaunchAttribute attr[2];
  attr[0].id = cudaLaunchAttributeClusterDimension;
  attr[0].val.clusterDim.y = 1;
  attr[0].val.clusterDim.z = 1;
  cfg.blockDim = dim3(kDThreads, 1, 1);
  cfg.dynamicSmemBytes = C::kSmemBytes;
  cfg.stream = s;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  // Split K over a cluster only while the clusters of all tiles are co-resident (one CTA
  // per SM): splits = the largest power of two <= 8 with tiles * splits <= SMs, that the
  // K range can feed and that the device can schedule.
  int splits = 1;
  while (splits * 2 <= kDMaxCluster && p.tiles_n * splits * 2 <= sms && splits * 2 <= p.num_kt)
    splits *= 2;
  for (; splits > 1; splits /= 2) {
    attr[0].val.clusterDim.x = splits;
    cfg.gridDim = dim3(p.tiles_n * splits, 1, 1);
    int ncl = 0;
    if (cudaOccupancyMaxActiveClusters(&ncl, gemm_decode_kernel<MPAD>, &cfg) == cudaSuccess &&
        ncl >= p.tiles_n)
      break;
    cudaGetLastError();
  }
  p.splits = splits;
  attr[0].val.clusterDim.x = splits;
  cfg.gridDim = dim3(p.tiles_n * splits, 1, 1);
  attr[1].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[1].val.programmaticStreamSerializationAllowed = 1;
  cfg.numAttrs = 2;
  cudaError_t e = cudaLaunchKernelEx(&cfg, gemm_decode_kernel<MPAD>, tw, tt, p);
  if (e != cudaSuccess) {
    set_err(err, std::string("decode launch: ") + cudaGetErrorString(e));
    return false;
  }
  return true;
}

bool decode_impl(const Nvfp4DeviceOperands& op, const uint8_t* sfa, const uint8_t* sfb, void* out,
                 const float* a_src, cudaStream_t s, std::string* err) {
  if (op.M > 128) {
    set_err(err, "decode kernel needs M <= 128");
    return false;
  }
  const int sms = device_sms(err);
  if (sms <= 0) return false;
  int dev = 0;
  cudaGetDevice(&dev);
  const int mpad = op.M <= 16 ? 16 : op.M <= 32 ? 32 : op.M <= 64 ? 64 : 128;
  DParams p;
  p.sfw = sfb;
  p.sft = sfa;
  p.out = out;
  p.M = op.M;
  p.N = op.N;
  p.K = op.K;
  p.alpha = op.a_global * op.b_global;
  p.out_bf16 = (op.d != nullptr && op.out_dtype == OutDType::BF16) ? 1 : 0;
  p.tiles_n = (op.N + 127) / 128;
  p.num_kt = 0;  // K-stages: set per stage depth in launch_decode
  p.ka = (op.K + 63) / 64;
  p.splits = 1;
  p.b_static = op.b_static ? 1 : 0;
  p.a_src = a_src;
  p.a_packed = const_cast<uint8_t*>(op.a_packed);
  p.a_g = op.a_global;
  {
    const int esz = p.out_bf16 ? 2 : 4;
    p.vec_out = ((static_cast<size_t>(op.N) * esz) % 16 == 0 &&
                 (reinterpret_cast<uintptr_t>(out) & 15) == 0) ? 1 : 0;
  }
  p.err_word = device_error_word(err);
  if (!p.err_word) return false;
  DecodeState* st = nullptr;
  {
    std::lock_guard<std::mutex> lk(g_dmu);
    if (static_cast<int>(g_dstate.size()) <= dev) g_dstate.resize(dev + 1);
    st = &g_dstate[dev];
  }
  CUtensorMap tw, tt;
  if (!operand_map(&tw, op.b_packed, op.N, op.K, 128, err)) return false;
  if (!operand_map(&tt, op.a_packed, op.M, op.K, mpad, err)) return false;
  switch (mpad) {
    case 16: return launch_decode<16>(tw, tt, p, sms, *st, 0, s, err);
    case 32: return launch_decode<32>(tw, tt, p, sms, *st, 1, s, err);
    case 64: return launch_decode<64>(tw, tt, p, sms, *st, 2, s, err);
    default: return launch_decode<128>(tw, tt, p, sms, *st, 3, s, err);
  }
}

}  // namespace

bool gemm_decode(const Nvfp4DeviceOperands& op, const uint8_t* sfa, const uint8_t* sfb, void* out,
                 cudaStream_t s, std::string* err) {
  return decode_impl(op, sfa, sfb, out, nullptr, s, err);
}

// Activation quantisation fused into the decode GEMM (no reference counterpart; the reference
// quantises on the host before every run, src/bench.cu:25-32): fp32 A [M][K] is quantised into
// op.a_packed and the tcgen05 scales `sfa` (both outputs, byte-identical to quantize()) and
// multiplied by B in one launch. M <= 128, K % 64 == 0, B scales in the tcgen05 layout. The
// kernel's grid barrier uses two counters in device memory: launches of this entry on one
// device must not overlap.
bool gemm_decode_quantize_a(const Nvfp4DeviceOperands& op, const float* a_src, uint8_t* sfa,
                            const uint8_t* sfb, void* out, cudaStream_t s, std::string* err) {
  if (!a_src || (reinterpret_cast<uintptr_t>(a_src) & 15) || op.K % 64 != 0 || op.M > 128 ||
      (reinterpret_cast<uintptr_t>(op.a_packed) & 15) || (reinterpret_cast<uintptr_t>(sfa) & 15)) {
    set_err(err, "fused quantisation needs a 16-byte aligned fp32 A, M <= 128, K % 64 == 0 and "
                 "16-byte aligned A outputs");
    return false;
  }
  return decode_impl(op, sfa, sfb, out, a_src, s, err);
}

}  // namespace nvfp4b200
