// gemm_decode.cu - weight-streaming NVFP4 GEMM for decode shapes (M <= 128 tokens).
//
// BASELINE's decode configurations (M in {16, 64, 128} tokens x a 14336 x 4096 or 4096 x
// 14336 weight) are HBM-bound: the weight B is read once and everything else is small. The
// general kernel tiles M by 128 rows, so at M = 16 it keeps at most N/128 CTAs busy and runs
// the MMA at 1/8 occupancy of its M; this kernel turns the problem around:
//   * the weight rows are the MMA's 128-row "A" side (D^T = B * A^T in TMEM, lane = weight
//     row n), the tokens its "B" side with N = M rounded up to 16..128;
//   * K is split over `splits` CTAs per 128-row weight tile so that about two CTAs per SM
//     stream weights (small shared memory, 256 TMEM columns, 2 CTAs per SM);
//   * partial sums go to an FP32 workspace; the last CTA of each tile (an atomic counter that
//     it resets) adds them in split order - deterministic - and writes C. With one split the
//     epilogue writes C directly.
// The epilogue needs no transpose: thread = weight row n holds the values of all tokens, so a
// warp stores 32 consecutive columns of C per token.
//
// Roles (320 threads): warp 0 TMA producer, warp 1 MMA issuer, warps 2..5 epilogue, warps
// 6..9 scale writers (tcgen05.st of each stage's scales into its TMEM slot, as in the general
// kernel). Bounded waits as everywhere (ptx.cuh).
#include <cuda.h>
#include <cuda_bf16.h>
#include <cuda_runtime.h>

#include <mutex>
#include <string>
#include <vector>

#include "gemm.h"
#include "internal.h"
#include "ptx.cuh"

namespace nvfp4b200 {
namespace {

constexpr int kDThreads = 320;
constexpr int kDMaxStages = 4;
constexpr int kDTmemCols = 256;   // accumulator [0, 128) + up to 4 stage slots of 32 columns
constexpr int kDSlotCols = 32;    // weight scales at +0 (4 per K-block), token scales at +16

struct DParams {
  const uint8_t* sfw;   // weight (B operand) scales, tcgen05 layout over N rows
  const uint8_t* sft;   // token (A operand) scales, tcgen05 layout over M rows
  void* out;
  float* ws;            // [splits][tiles_n][mpad][128] partial sums (splits > 1)
  int* counters;        // [tiles_n], zero between calls
  int M, N, K;
  float alpha;
  int out_bf16;
  int tiles_n, splits, num_kt, ka;
  uint32_t* err_word;
};

template <int MPAD>
struct DCfg {
  // Stages: 4, or 3 for 64-token tiles so that two CTAs still fit one SM's shared memory.
  static constexpr int kStages = MPAD == 64 ? 3 : kDMaxStages;
  static constexpr int kWBytes = 128 * 128;           // 128 weight rows x 256 FP4
  static constexpr int kTBytes = MPAD * 128;          // MPAD token rows x 256 FP4
  static constexpr int kSfBytes = 4 * 512;            // one 128-row atom per K-block
  static constexpr int kStageBytes = kWBytes + kTBytes + 2 * kSfBytes;
  static constexpr int kSmemBytes = 1024 + kStages * kStageBytes + 256;
  static constexpr int kMinBlocks = MPAD <= 64 ? 2 : 1;
  static_assert(kStages * kDSlotCols + 128 <= kDTmemCols, "TMEM budget");
};

__device__ __forceinline__ void store_out(const DParams& p, int m, int n, float v) {
  if (p.out_bf16)
    reinterpret_cast<__nv_bfloat16*>(p.out)[static_cast<size_t>(m) * p.N + n] = __float2bfloat16_rn(v);
  else
    reinterpret_cast<float*>(p.out)[static_cast<size_t>(m) * p.N + n] = v;
}

template <int MPAD>
__global__ void __launch_bounds__(kDThreads, DCfg<MPAD>::kMinBlocks)
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
  uint64_t* bars = reinterpret_cast<uint64_t*>(sSFT + C::kStages * C::kSfBytes);
  uint64_t* full = bars;                 // operand bytes + producer + 4 scale writers
  uint64_t* empty = full + C::kStages;     // stage (smem and scale slot) consumed
  uint64_t* sfd = empty + C::kStages;      // scale bytes landed
  uint64_t* acc_full = sfd + C::kStages;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(acc_full + 1);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);
  int* last_flag = const_cast<int*>(abort_flag) + 1;

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int tn = blockIdx.x % p.tiles_n, ks = blockIdx.x / p.tiles_n;
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
    *last_flag = 0;
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

  if (warp == 0) {
    if (lane == 0) {
      bool ok = true;
      int i = 0;
      for (int kt = kt0; kt < kt1; ++kt, ++i) {
        const int s = i % C::kStages;
        const uint32_t j = static_cast<uint32_t>(i / C::kStages);
        if (!mbar_wait(smem_u32(&empty[s]), (j & 1u) ^ 1u, abort_flag, p.err_word,
                       kErrWaitSmemEmpty)) {
          ok = false;
          break;
        }
        int nkb = p.ka - kt * 4;
        if (nkb > 4) nkb = 4;
        const uint32_t sfb = static_cast<uint32_t>(nkb) * 512u;
        const uint32_t db = smem_u32(&sfd[s]);
        mbar_arrive_expect_tx(db, 2 * sfb);
        bulk_load(smem_u32(sSFW + s * C::kSfBytes),
                  p.sfw + (static_cast<size_t>(tn) * p.ka + kt * 4) * 512, sfb, db);
        bulk_load(smem_u32(sSFT + s * C::kSfBytes), p.sft + static_cast<size_t>(kt) * 4 * 512,
                  sfb, db);
        const uint32_t fb = smem_u32(&full[s]);
        mbar_arrive_expect_tx(fb, C::kWBytes + C::kTBytes);
        tma_load_2d(smem_u32(sW + s * C::kWBytes), &tmap_w, kt * 128, tn * 128, fb);
        tma_load_2d(smem_u32(sT + s * C::kTBytes), &tmap_t, kt * 128, 0, fb);
      }
      if (!ok) {
        for (int back = 1; back <= C::kStages && i - back >= 0; ++back) {
          const int f = i - back;
          volatile int never = 0;
          mbar_wait(smem_u32(&sfd[f % C::kStages]), static_cast<uint32_t>(f / C::kStages) & 1u,
                    &never, p.err_word, kErrWaitDrain);
        }
      }
    }
  } else if (warp == 1) {
    if (lane == 0) {
      const uint32_t idesc = make_idesc_mxf4nvf4(128, MPAD);
      bool ok = true, issued = false;
      int i = 0;
      for (int kt = kt0; kt < kt1; ++kt, ++i) {
        const int s = i % C::kStages;
        const uint32_t j = static_cast<uint32_t>(i / C::kStages);
        if (!mbar_spin_wait<false>(smem_u32(&full[s]), j & 1u, abort_flag, p.err_word,
                                   kErrWaitTmaFull)) {
          ok = false;
          break;
        }
        tc_fence_after();
        int nkb = p.ka - kt * 4;
        if (nkb > 4) nkb = 4;
        const uint64_t ad0 = make_sdesc(smem_u32(sW + s * C::kWBytes), 16, 1024, 2);
        const uint64_t bd0 = make_sdesc(smem_u32(sT + s * C::kTBytes), 16, 1024, 2);
        const uint32_t sf_t = tmem_base + 128 + s * kDSlotCols;
        for (int kb = 0; kb < nkb; ++kb)
          tc_mma_mxf4nvf4(tmem_base, ad0 + 2 * kb, bd0 + 2 * kb, idesc, sf_t + kb * 4,
                          sf_t + 16 + kb * 4, (i > 0 || kb > 0) ? 1u : 0u);
        issued = true;
        tc_commit(smem_u32(&empty[s]));
      }
      if (ok) {
        tc_commit(smem_u32(acc_full));
      } else if (issued) {
        tc_commit(smem_u32(acc_full));
        volatile int never = 0;
        mbar_wait(smem_u32(acc_full), 0, &never, p.err_word, kErrWaitDrain);
      }
    }
  } else if (warp >= 6) {
    // Scale writers: weight atom -> slot +0, token atom -> slot +16 (4 words per K-block).
    const int q = warp & 3;
    const uint32_t lane_base = tmem_base + (static_cast<uint32_t>(q * 32) << 16);
    int i = 0;
    for (int kt = kt0; kt < kt1; ++kt, ++i) {
      const int s = i % C::kStages;
      const uint32_t j = static_cast<uint32_t>(i / C::kStages);
      if (!mbar_wait(smem_u32(&sfd[s]), j & 1u, abort_flag, p.err_word, kErrWaitTmaFull)) break;
      uint32_t vw[16], vt[16];
#pragma unroll
      for (int kb = 0; kb < 4; ++kb) {
        const uint4 w = *reinterpret_cast<const uint4*>(sSFW + s * C::kSfBytes + kb * 512 + lane * 16);
        const uint4 t = *reinterpret_cast<const uint4*>(sSFT + s * C::kSfBytes + kb * 512 + lane * 16);
        vw[4 * kb] = w.x; vw[4 * kb + 1] = w.y; vw[4 * kb + 2] = w.z; vw[4 * kb + 3] = w.w;
        vt[4 * kb] = t.x; vt[4 * kb + 1] = t.y; vt[4 * kb + 2] = t.z; vt[4 * kb + 3] = t.w;
      }
      if (!mbar_wait(smem_u32(&empty[s]), (j & 1u) ^ 1u, abort_flag, p.err_word, kErrWaitSfEmpty))
        break;
      tc_fence_after();
      const uint32_t sf_t = lane_base + 128 + s * kDSlotCols;
      tmem_st_32x32b_x16(sf_t, vw);
      tmem_st_32x32b_x16(sf_t + 16, vt);
      tc_wait_st();
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(smem_u32(&full[s]));
    }
  } else {
    // Epilogue: thread = weight row n (TMEM lane), registers = tokens.
    const int q = warp & 3;
    const int n_local = q * 32 + lane;
    const int n = tn * 128 + n_local;
    bool ok = mbar_wait(smem_u32(acc_full), 0, abort_flag, p.err_word, kErrWaitAccFull);
    tc_fence_after();
    const uint32_t acc_t = tmem_base + (static_cast<uint32_t>(q * 32) << 16);
    if (p.splits == 1) {
#pragma unroll
      for (int c0 = 0; c0 < MPAD; c0 += 32) {
        uint32_t r[32];
        tmem_ld_32x32b_x32(acc_t + c0, r);
        tc_wait_ld();
        if (ok && n < p.N) {
#pragma unroll
          for (int jj = 0; jj < 32; ++jj)
            if (c0 + jj < p.M) store_out(p, c0 + jj, n, __uint_as_float(r[jj]) * p.alpha);
        }
      }
    } else {
      float* part = p.ws + (static_cast<size_t>(ks) * p.tiles_n + tn) * MPAD * 128;
#pragma unroll
      for (int c0 = 0; c0 < MPAD; c0 += 32) {
        uint32_t r[32];
        tmem_ld_32x32b_x32(acc_t + c0, r);
        tc_wait_ld();
#pragma unroll
        for (int jj = 0; jj < 32; ++jj)
          if (c0 + jj < MPAD) __stcg(part + (c0 + jj) * 128 + n_local, __uint_as_float(r[jj]));
      }
      __threadfence();
      asm volatile("bar.sync 1, 128;" ::: "memory");
      if (q == (2 & 3) && lane == 0) {
        const int old = atomicAdd(&p.counters[tn], 1);
        *last_flag = (old == p.splits - 1) ? 1 : 0;
      }
      asm volatile("bar.sync 1, 128;" ::: "memory");
    }
  }

  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  if (warp == 1) tmem_dealloc(tmem_base, kDTmemCols);

  if (p.splits > 1 && *last_flag) {
    // The last CTA of this weight tile adds the splits' partial sums in split order. All 320
    // threads take (token, row) pairs in turn; each pair's loads are independent of the
    // stores (restrict) and issue together.
    __threadfence();
    const float* __restrict__ ws = p.ws + static_cast<size_t>(tn) * MPAD * 128;
    const size_t split_stride = static_cast<size_t>(p.tiles_n) * MPAD * 128;
    const int total = p.M * 128;
    for (int idx = threadIdx.x; idx < total; idx += kDThreads) {
      float acc = 0.0f;
      for (int k2 = 0; k2 < p.splits; ++k2) acc += __ldcg(ws + k2 * split_stride + idx);
      const int m = idx >> 7, nn = tn * 128 + (idx & 127);
      if (nn < p.N) store_out(p, m, nn, acc * p.alpha);
    }
    if (threadIdx.x == 0) p.counters[tn] = 0;
  }
}

struct DecodeWs {
  float* ws = nullptr;
  size_t ws_bytes = 0;
  int* counters = nullptr;
  int n_counters = 0;
  bool attr[4] = {false, false, false, false};
};
std::mutex g_dmu;
std::vector<DecodeWs> g_dws;

template <int MPAD>
bool launch_decode(const CUtensorMap& tw, const CUtensorMap& tt, const DParams& p, DecodeWs& w,
                   int idx, cudaStream_t s, std::string* err) {
  using C = DCfg<MPAD>;
  if (!w.attr[idx]) {
    cudaError_t e = cudaFuncSetAttribute(gemm_decode_kernel<MPAD>,
                                         cudaFuncAttributeMaxDynamicSharedMemorySize, C::kSmemBytes);
    if (e != cudaSuccess) {
      set_err(err, std::string("cudaFuncSetAttribute (decode): ") + cudaGetErrorString(e));
      return false;
    }
    w.attr[idx] = true;
  }
  gemm_decode_kernel<MPAD><<<p.tiles_n * p.splits, kDThreads, C::kSmemBytes, s>>>(tw, tt, p);
  cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) {
    set_err(err, std::string("decode launch: ") + cudaGetErrorString(e));
    return false;
  }
  return true;
}

}  // namespace

bool gemm_decode(const Nvfp4DeviceOperands& op, const uint8_t* sfa, const uint8_t* sfb, void* out,
                 cudaStream_t s, std::string* err) {
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
  p.num_kt = (op.K + 255) / 256;
  p.ka = (op.K + 63) / 64;
  const int per_sm = mpad <= 64 ? 2 : 1;
  // One wave: as many K splits as keep tiles_n * splits within the co-resident CTA count.
  int splits = (per_sm * sms) / p.tiles_n;
  if (splits > p.num_kt) splits = p.num_kt;
  if (splits < 1) splits = 1;
  p.splits = splits;
  p.err_word = device_error_word(err);
  if (!p.err_word) return false;
  {
    std::lock_guard<std::mutex> lk(g_dmu);
    if (static_cast<int>(g_dws.size()) <= dev) g_dws.resize(dev + 1);
    DecodeWs& w = g_dws[dev];
    const size_t need = static_cast<size_t>(splits) * p.tiles_n * mpad * 128 * sizeof(float);
    if (splits > 1 && w.ws_bytes < need) {
      if (w.ws) cudaFree(w.ws);
      w.ws = nullptr;
      w.ws_bytes = 0;
      if (cudaMalloc(&w.ws, need) != cudaSuccess) {
        set_err(err, "cudaMalloc of the decode workspace failed");
        return false;
      }
      w.ws_bytes = need;
    }
    if (w.n_counters < p.tiles_n) {
      if (w.counters) cudaFree(w.counters);
      w.counters = nullptr;
      w.n_counters = 0;
      if (cudaMalloc(&w.counters, sizeof(int) * p.tiles_n) != cudaSuccess ||
          cudaMemset(w.counters, 0, sizeof(int) * p.tiles_n) != cudaSuccess) {
        set_err(err, "cudaMalloc of the decode counters failed");
        return false;
      }
      w.n_counters = p.tiles_n;
    }
    p.ws = w.ws;
    p.counters = w.counters;
  }
  CUtensorMap tw, tt;
  if (!operand_map(&tw, op.b_packed, op.N, op.K, 128, err)) return false;
  if (!operand_map(&tt, op.a_packed, op.M, op.K, mpad, err)) return false;
  DecodeWs& w = g_dws[dev];
  switch (mpad) {
    case 16: return launch_decode<16>(tw, tt, p, w, 0, s, err);
    case 32: return launch_decode<32>(tw, tt, p, w, 1, s, err);
    case 64: return launch_decode<64>(tw, tt, p, w, 2, s, err);
    default: return launch_decode<128>(tw, tt, p, w, 3, s, err);
  }
}

}  // namespace nvfp4b200
