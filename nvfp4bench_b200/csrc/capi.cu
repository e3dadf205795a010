// capi.cu - the C ABI (include/nvfp4_b200.h) over the engine's C++ entry points, and the
// reference's GB10-only backend slots, which this engine does not build.
#include <cuda_runtime.h>

#include <cstring>
#include <string>

#include "gemm.h"
#include "internal.h"
#include "nvfp4_b200.h"

namespace {

int fail(int code, const std::string& msg, char* err, size_t errlen) {
  if (err && errlen) {
    size_t n = msg.size() < errlen - 1 ? msg.size() : errlen - 1;
    std::memcpy(err, msg.data(), n);
    err[n] = '\0';
  }
  return code;
}

int ok(char* err, size_t errlen) {
  if (err && errlen) err[0] = '\0';
  return NVFP4_B200_OK;
}

// Argument errors are EINVAL; anything that mentions CUDA is ECUDA.
int classify(const std::string& msg) {
  if (msg.find("sm_100") != std::string::npos) return NVFP4_B200_EUNSUPPORTED;
  if (msg.find("not built") != std::string::npos || msg.find("not supported") != std::string::npos)
    return NVFP4_B200_EUNSUPPORTED;
  if (msg.find("cuda") != std::string::npos || msg.find("CUDA") != std::string::npos ||
      msg.find("launch") != std::string::npos || msg.find("failed") != std::string::npos)
    return NVFP4_B200_ECUDA;
  return NVFP4_B200_EINVAL;
}

}  // namespace

// The reference's GB10 backends (src/gemm_stub.cu, src/gemm_cutlass.cu, src/gemm_custom.cu)
// use sm_120a warp-level MMAs that do not exist on sm_100a; like the reference's own
// "not built" stubs (src/gemm_custom.cu:18-23) they report that and return false.
bool launch_gemm_stub(const Nvfp4DeviceOperands&, cudaStream_t, std::string* err) {
  if (err) *err = "stub backend not built (GB10 reference backend; use --kernel b200)";
  return false;
}
bool launch_gemm_cutlass(const Nvfp4DeviceOperands&, cudaStream_t, std::string* err) {
  if (err) *err = "cutlass backend not built (GB10 reference backend; use --kernel b200)";
  return false;
}
bool launch_gemm_custom(const Nvfp4DeviceOperands&, cudaStream_t, std::string* err) {
  if (err) *err = "custom backend not built (GB10 reference backend; use --kernel b200)";
  return false;
}

extern "C" {

int nvfp4_b200_gemm(const Nvfp4GemmArgs* a, void* stream, char* err, size_t errlen) {
  if (!a) return fail(NVFP4_B200_EINVAL, "null args", err, errlen);
  Nvfp4DeviceOperands op;
  op.a_packed = static_cast<const uint8_t*>(a->a_packed);
  op.a_scales = static_cast<const uint8_t*>(a->a_scales);
  op.a_global = a->a_global;
  op.b_packed = static_cast<const uint8_t*>(a->b_packed);
  op.b_scales = static_cast<const uint8_t*>(a->b_scales);
  op.b_global = a->b_global;
  op.M = a->M;
  op.N = a->N;
  op.K = a->K;
  if (a->mode != NVFP4_MODE_DENSE && a->mode != NVFP4_MODE_SPARSE24)
    return fail(NVFP4_B200_EINVAL, "unknown mode", err, errlen);
  if (a->sf_layout != NVFP4_SF_CANONICAL && a->sf_layout != NVFP4_SF_TCGEN05)
    return fail(NVFP4_B200_EINVAL, "unknown sf_layout", err, errlen);
  if (a->out_dtype != NVFP4_OUT_F32 && a->out_dtype != NVFP4_OUT_BF16 &&
      a->out_dtype != NVFP4_OUT_NVFP4)
    return fail(NVFP4_B200_EINVAL, "unknown out_dtype", err, errlen);
  op.mode = a->mode == NVFP4_MODE_SPARSE24 ? GemmMode::Sparse : GemmMode::Dense;
  op.sf_layout = a->sf_layout == NVFP4_SF_TCGEN05 ? SfLayout::Tcgen05 : SfLayout::Canonical;
  op.out_dtype = a->out_dtype == NVFP4_OUT_BF16    ? OutDType::BF16
                 : a->out_dtype == NVFP4_OUT_NVFP4 ? OutDType::NVFP4
                                                   : OutDType::F32;
  if (op.out_dtype == OutDType::NVFP4) {
    if (a->c_sf_layout != NVFP4_SF_CANONICAL && a->c_sf_layout != NVFP4_SF_TCGEN05)
      return fail(NVFP4_B200_EINVAL, "unknown c_sf_layout", err, errlen);
    op.d_scales = static_cast<uint8_t*>(a->c_scales);
    op.d_global = a->c_global;
    op.d_sf_layout = a->c_sf_layout == NVFP4_SF_TCGEN05 ? SfLayout::Tcgen05 : SfLayout::Canonical;
  }
  op.d = a->c;
  op.a_meta = static_cast<const uint8_t*>(a->a_meta);
  op.cta_group = a->cta_group;
  op.tile_n = a->tile_n;
  op.b_static = (a->flags & NVFP4_FLAG_B_STATIC) != 0;
  // Checked before any CUDA call (the engine checks them again with the device-side rules).
  if (a->ldc != 0 && a->ldc < a->N) return fail(NVFP4_B200_EINVAL, "ldc must be at least N", err, errlen);
  if (a->n_peers < 0 || a->n_peers > 7 || (a->n_peers > 0 && !a->c_peers))
    return fail(NVFP4_B200_EINVAL, "n_peers must be 0..7 with a c_peers array", err, errlen);
  op.ldd = a->ldc;
  op.d_peers = a->c_peers;
  op.n_peers = a->n_peers;
  std::string e;
  if (!launch_gemm_b200(op, static_cast<cudaStream_t>(stream), &e))
    return fail(classify(e), e, err, errlen);
  return ok(err, errlen);
}

int nvfp4_b200_gemm_quantize_a(const Nvfp4GemmArgs* a, const float* a_src, void* stream, char* err,
                               size_t errlen) {
  if (!a || !a_src) return fail(NVFP4_B200_EINVAL, "null args or a_src", err, errlen);
  if (a->mode != NVFP4_MODE_DENSE)
    return fail(NVFP4_B200_EINVAL, "the fused quantisation GEMM is dense only", err, errlen);
  if (a->sf_layout != NVFP4_SF_TCGEN05)
    return fail(NVFP4_B200_EINVAL, "the fused quantisation GEMM takes tcgen05-layout scales "
                "(a_scales is written, b_scales read)", err, errlen);
  if (!a->a_packed || !a->a_scales)
    return fail(NVFP4_B200_EINVAL, "a_packed and a_scales (outputs) must be given", err, errlen);
  if (a->M <= 0 || a->K <= 0 || a->K % 16 != 0)
    return fail(NVFP4_B200_EINVAL, "M must be positive and K a multiple of 16", err, errlen);
  bool fused = a->M <= 128 && a->K % 64 == 0 && a->cta_group == 0 && a->tile_n == 0 &&
               (a->out_dtype == NVFP4_OUT_F32 || a->out_dtype == NVFP4_OUT_BF16) &&
               (a->ldc == 0 || a->ldc == a->N) && a->n_peers == 0;
  if (fused) {
    // The single launch meets at a grid barrier, which costs more than the second launch when
    // the decode kernel splits K over thread-block clusters (fewer weight tiles than half the
    // SMs; measured: M=16 down-proj 19.8 us fused, 16.4 us as two launches; up-proj M=16
    // 13.8 us fused, 14.4 us as two). Fuse only when there is no split.
    std::string e0;
    const int sms = nvfp4b200::device_sms(&e0);
    if (sms <= 0) return fail(NVFP4_B200_ECUDA, e0, err, errlen);
    fused = static_cast<long>((a->N + 127) / 128) * 2 > sms;
  }
  const cudaStream_t s = static_cast<cudaStream_t>(stream);
  std::string e;
  if (!fused) {
    // Any other shape: the standalone quantiser, then the GEMM, on the same stream.
    if (!nvfp4b200::quantize(a_src, a->M, a->K, a->a_global, static_cast<uint8_t*>(const_cast<void*>(a->a_packed)),
                             nullptr, static_cast<uint8_t*>(const_cast<void*>(a->a_scales)), s, &e))
      return fail(classify(e), e, err, errlen);
    return nvfp4_b200_gemm(a, stream, err, errlen);
  }
  const int cc = nvfp4b200::device_cc_major(&e);
  if (cc == 0) return fail(NVFP4_B200_ECUDA, e, err, errlen);
  if (cc != 10) return fail(NVFP4_B200_EUNSUPPORTED, "the b200 backend needs an sm_100 device", err, errlen);
  if (!a->b_packed || !a->b_scales || !a->c) return fail(NVFP4_B200_EINVAL, "null operand pointer", err, errlen);
  if ((reinterpret_cast<uintptr_t>(a->b_packed) | reinterpret_cast<uintptr_t>(a->b_scales)) & 15)
    return fail(NVFP4_B200_EINVAL, "B and its scales must be 16-byte aligned", err, errlen);
  Nvfp4DeviceOperands op;
  op.a_packed = static_cast<const uint8_t*>(a->a_packed);
  op.a_scales = static_cast<const uint8_t*>(a->a_scales);
  op.a_global = a->a_global;
  op.b_packed = static_cast<const uint8_t*>(a->b_packed);
  op.b_scales = static_cast<const uint8_t*>(a->b_scales);
  op.b_global = a->b_global;
  op.M = a->M;
  op.N = a->N;
  op.K = a->K;
  op.sf_layout = SfLayout::Tcgen05;
  op.out_dtype = a->out_dtype == NVFP4_OUT_BF16 ? OutDType::BF16 : OutDType::F32;
  op.d = a->c;
  op.b_static = (a->flags & NVFP4_FLAG_B_STATIC) != 0;
  if (!nvfp4b200::gemm_decode_quantize_a(op, a_src, static_cast<uint8_t*>(const_cast<void*>(a->a_scales)),
                                         static_cast<const uint8_t*>(a->b_scales), a->c, s, &e))
    return fail(classify(e), e, err, errlen);
  return ok(err, errlen);
}

int nvfp4_b200_gemm_noalloc(const Nvfp4GemmArgs* a, void* stream, char* err, size_t errlen) {
  if (!a) return fail(NVFP4_B200_EINVAL, "null args", err, errlen);
  if (a->mode != NVFP4_MODE_DENSE)
    return fail(NVFP4_B200_EINVAL, "the no-alloc GEMM supports dense mode only", err, errlen);
  if (a->sf_layout != NVFP4_SF_CANONICAL)
    return fail(NVFP4_B200_EINVAL, "the no-alloc GEMM takes canonical scales", err, errlen);
  if (a->out_dtype == NVFP4_OUT_NVFP4)
    return fail(NVFP4_B200_EUNSUPPORTED,
                "NVFP4 output is not supported by the no-alloc GEMM (FP32 or BF16 only)", err, errlen);
  if (a->out_dtype != NVFP4_OUT_F32 && a->out_dtype != NVFP4_OUT_BF16)
    return fail(NVFP4_B200_EINVAL, "unknown out_dtype", err, errlen);
  Nvfp4DeviceOperands op;
  op.a_packed = static_cast<const uint8_t*>(a->a_packed);
  op.a_scales = static_cast<const uint8_t*>(a->a_scales);
  op.a_global = a->a_global;
  op.b_packed = static_cast<const uint8_t*>(a->b_packed);
  op.b_scales = static_cast<const uint8_t*>(a->b_scales);
  op.b_global = a->b_global;
  op.M = a->M;
  op.N = a->N;
  op.K = a->K;
  op.mode = GemmMode::Dense;
  op.sf_layout = SfLayout::Canonical;
  op.out_dtype = a->out_dtype == NVFP4_OUT_BF16 ? OutDType::BF16 : OutDType::F32;
  if (a->n_peers != 0)
    return fail(NVFP4_B200_EINVAL, "the no-alloc GEMM does not write peer outputs", err, errlen);
  op.d = a->c;
  op.ldd = a->ldc;
  op.cta_group = a->cta_group;
  op.tile_n = a->tile_n;
  std::string e;
  if (!nvfp4b200::gemm_noalloc(op, static_cast<cudaStream_t>(stream), &e))
    return fail(classify(e), e, err, errlen);
  return ok(err, errlen);
}

size_t nvfp4_b200_gemm_noalloc_scratch_bytes(void) { return nvfp4b200::noalloc_scratch_bytes(); }

int nvfp4_b200_quantize(const float* src, int rows, int cols, float global_scale, void* packed,
                        void* scales, void* scales_tc, void* stream, char* err, size_t errlen) {
  std::string e;
  if (!nvfp4b200::quantize(src, rows, cols, global_scale, static_cast<uint8_t*>(packed),
                           static_cast<uint8_t*>(scales), static_cast<uint8_t*>(scales_tc),
                           static_cast<cudaStream_t>(stream), &e))
    return fail(classify(e), e, err, errlen);
  return ok(err, errlen);
}

int nvfp4_b200_dequantize(const void* packed, const void* scales, int rows, int cols,
                          float global_scale, float* out, void* stream, char* err, size_t errlen) {
  std::string e;
  if (!nvfp4b200::dequantize(static_cast<const uint8_t*>(packed), static_cast<const uint8_t*>(scales),
                             rows, cols, global_scale, out, static_cast<cudaStream_t>(stream), &e))
    return fail(classify(e), e, err, errlen);
  return ok(err, errlen);
}

int nvfp4_b200_quantize_ex(const float* src, int rows, int cols, float global_scale, int block,
                           void* packed, void* scales, void* scales_tc, void* stream, char* err,
                           size_t errlen) {
  std::string e;
  if (!nvfp4b200::quantize_block(src, rows, cols, global_scale, block, static_cast<uint8_t*>(packed),
                                 static_cast<uint8_t*>(scales), static_cast<uint8_t*>(scales_tc),
                                 static_cast<cudaStream_t>(stream), &e))
    return fail(classify(e), e, err, errlen);
  return ok(err, errlen);
}

int nvfp4_b200_dequantize_ex(const void* packed, const void* scales, int rows, int cols,
                             float global_scale, int block, float* out, void* stream, char* err,
                             size_t errlen) {
  std::string e;
  if (!nvfp4b200::dequantize_block(static_cast<const uint8_t*>(packed),
                                   static_cast<const uint8_t*>(scales), rows, cols, global_scale,
                                   block, out, static_cast<cudaStream_t>(stream), &e))
    return fail(classify(e), e, err, errlen);
  return ok(err, errlen);
}

int nvfp4_b200_sparse_meta(int rows, int K, uint64_t seed, void* meta, void* stream, char* err,
                           size_t errlen) {
  std::string e;
  if (!nvfp4b200::sparse_meta(rows, K, seed, static_cast<uint8_t*>(meta),
                              static_cast<cudaStream_t>(stream), &e))
    return fail(classify(e), e, err, errlen);
  return ok(err, errlen);
}

int nvfp4_b200_sparse_prune(float* a, int rows, int K, const void* meta, void* stream, char* err,
                            size_t errlen) {
  std::string e;
  if (!nvfp4b200::sparse_prune(a, rows, K, static_cast<const uint8_t*>(meta),
                               static_cast<cudaStream_t>(stream), &e))
    return fail(classify(e), e, err, errlen);
  return ok(err, errlen);
}

int nvfp4_b200_sparse_compress(const void* packed, int rows, int K, const void* meta, void* values,
                               void* stream, char* err, size_t errlen) {
  std::string e;
  if (!nvfp4b200::sparse_compress(static_cast<const uint8_t*>(packed), rows, K,
                                  static_cast<const uint8_t*>(meta), static_cast<uint8_t*>(values),
                                  static_cast<cudaStream_t>(stream), &e))
    return fail(classify(e), e, err, errlen);
  return ok(err, errlen);
}

int nvfp4_b200_fill_uniform(float* out, int rows, int cols, uint64_t seed, void* stream, char* err,
                            size_t errlen) {
  if (rows < 0 || cols < 0) return fail(NVFP4_B200_EINVAL, "negative size", err, errlen);
  std::string e;
  if (!nvfp4b200::fill_uniform(out, static_cast<size_t>(rows) * cols, seed,
                               static_cast<cudaStream_t>(stream), &e))
    return fail(classify(e), e, err, errlen);
  return ok(err, errlen);
}

int nvfp4_b200_fill_normal(float* out, int rows, int cols, uint64_t seed, void* stream, char* err,
                           size_t errlen) {
  if (rows < 0 || cols < 0) return fail(NVFP4_B200_EINVAL, "negative size", err, errlen);
  std::string e;
  if (!nvfp4b200::fill_normal(out, static_cast<size_t>(rows) * cols, seed,
                              static_cast<cudaStream_t>(stream), &e))
    return fail(classify(e), e, err, errlen);
  return ok(err, errlen);
}

size_t nvfp4_b200_sf_tcgen05_bytes(int rows, int K) {
  if (rows <= 0 || K <= 0) return 0;
  return nvfp4b200::sf_tcgen05_bytes(rows, K);
}

int nvfp4_b200_sf_to_tcgen05(const void* scales, int rows, int K, void* out, void* stream,
                             char* err, size_t errlen) {
  std::string e;
  if (!nvfp4b200::sf_to_tcgen05(static_cast<const uint8_t*>(scales), rows, K,
                                static_cast<uint8_t*>(out), static_cast<cudaStream_t>(stream), &e))
    return fail(classify(e), e, err, errlen);
  return ok(err, errlen);
}

int nvfp4_b200_measure_bandwidth(int kind, const void* src, void* dst, const void* src2,
                                 size_t bytes, int iters, double* gbs, void* stream, char* err,
                                 size_t errlen) {
  std::string e;
  if (!nvfp4b200::measure_bandwidth(kind, src, dst, src2, bytes, iters, gbs,
                                    static_cast<cudaStream_t>(stream), &e))
    return fail(classify(e), e, err, errlen);
  return ok(err, errlen);
}

int nvfp4_b200_peak(int n, int ctas, int iters, int reps, double* tflops, void* stream, char* err,
                    size_t errlen) {
  std::string e;
  if (!nvfp4b200::peak_ladder(n, ctas, iters, reps, tflops, static_cast<cudaStream_t>(stream), &e))
    return fail(classify(e), e, err, errlen);
  return ok(err, errlen);
}

int nvfp4_b200_peak_ex(int n, int cta_group, int units, int iters, int reps, uint32_t seed,
                       int sustained, int sparse, double* tflops, double* sm_mhz, void* stream,
                       char* err, size_t errlen) {
  std::string e;
  const nvfp4b200::PeakOptions o{n, cta_group, units, iters, reps, seed, sustained, sparse};
  if (!nvfp4b200::peak_ladder_ex(o, tflops, sm_mhz, static_cast<cudaStream_t>(stream), &e))
    return fail(classify(e), e, err, errlen);
  return ok(err, errlen);
}

int nvfp4_b200_device_error(int clear, uint32_t* word, char* err, size_t errlen) {
  std::string e;
  uint32_t* ew = nvfp4b200::device_error_word(&e);
  if (!ew) return fail(NVFP4_B200_ECUDA, e, err, errlen);
  if (cudaDeviceSynchronize() != cudaSuccess)
    return fail(NVFP4_B200_ECUDA, "cudaDeviceSynchronize failed", err, errlen);
  uint32_t w = 0;
  if (cudaMemcpy(&w, ew, sizeof(w), cudaMemcpyDeviceToHost) != cudaSuccess)
    return fail(NVFP4_B200_ECUDA, "reading the device error word failed", err, errlen);
  if (clear && cudaMemset(ew, 0, sizeof(uint32_t)) != cudaSuccess)
    return fail(NVFP4_B200_ECUDA, "clearing the device error word failed", err, errlen);
  if (word) *word = w;
  return ok(err, errlen);
}

int nvfp4_b200_wait_selftest(uint64_t limit_ns, uint32_t* word, char* err, size_t errlen) {
  std::string e;
  if (!nvfp4b200::wait_selftest(limit_ns, &e)) return fail(classify(e), e, err, errlen);
  return nvfp4_b200_device_error(1, word, err, errlen);
}

const char* nvfp4_b200_version(void) { return "nvfp4-b200 0.1.0 (sm_100a tcgen05)"; }

}  // extern "C"
