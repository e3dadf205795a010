// main.cpp - nvfp4bench: the C++ benchmark harness of the engine.
//
// Counterpart of the reference's CLI and harness (src/main.cu:14-135, src/bench.cu:25-187)
// driving the backends through launch_gemm(KernelKind, ...) (include/gemm.h). Same flags, same
// per-launch event timing (burst = min, sustained = median), same table / CSV / JSON reports;
// operands are generated and quantised on the GPU (the reference quantises on the host),
// B is N x K, and --validate compares with a GPU naive FP32 GEMM on the dequantised operands
// (the reference's oracle design, src/reference.cu:9-17) using the engine's criterion
// max|err| <= tol * max|C_ref| next to the reference's max relative error.
#include <cuda_runtime.h>
#include <dlfcn.h>

#include <algorithm>
#include <cmath>
#include <cstdio>
#include <cstring>
#include <fstream>
#include <string>
#include <vector>

#include "common.h"
#include "gemm.h"
#include "internal.h"

namespace {

struct Config {
  int iters = 50;
  int warmup = 10;
  bool validate = false;
  double tol = 1e-3;
  uint64_t seed = 1234;
  bool normal = true;
  bool bf16 = false;
  bool tcgen05_sf = true;
  int cta_group = 0;
  int tile_n = 0;
};

struct Dev {
  int id = 0;
  std::string name;
  int sms = 0;
  double peak_tflops = 0.0;  // measured tcgen05 ladder (filled by --peak or lazily)
};

void usage(const char* prog) {
  std::printf(
      "nvfp4bench (B200 engine) - NVFP4 block-scaled GEMM benchmark on sm_100a\n\n"
      "Usage: %s [options]\n\n"
      "  --kernel  b200|stub|cutlass|custom|all  backends (default: b200; the others are the\n"
      "                                          reference's GB10 backends, not built here)\n"
      "  --mode    dense|sparse|both      (default dense)\n"
      "  --m N --n N --k N                single GEMM size (default 4096x14336x4096)\n"
      "  --sweep                          preset sizes (the reference's sweep + BASELINE configs)\n"
      "  --iters N / --warmup N           timed / warm-up launches (default 50 / 10)\n"
      "  --validate [--tol F]             check against the FP32 oracle (default tol 1e-3 of max|C|)\n"
      "  --dist normal|uniform            operand distribution (uniform = reference generator)\n"
      "  --out f32|bf16                   output type (default f32, as the reference)\n"
      "  --sf tcgen05|canonical           scale layout handed to the backend (default tcgen05)\n"
      "  --cta-group 0|1|2 --tile-n N     kernel selection (0 = heuristic)\n"
      "  --peak                           tcgen05 FP4 throughput ladder (measured compute roof)\n"
      "  --bandwidth                      HBM roof (copy / read / triad)\n"
      "  --device N --csv FILE --json FILE\n",
      prog);
}

bool eq(const char* a, const char* b) { return std::strcmp(a, b) == 0; }

#define CK(x)                                                                         \
  do {                                                                                \
    cudaError_t e_ = (x);                                                             \
    if (e_ != cudaSuccess) {                                                          \
      std::fprintf(stderr, "CUDA error %s at %s:%d\n", cudaGetErrorString(e_), __FILE__, \
                   __LINE__);                                                         \
      std::exit(1);                                                                   \
    }                                                                                 \
  } while (0)

struct Operand {
  uint8_t* packed = nullptr;     // dense [rows][K/2]; sparse A: kept values [rows][K/4]
  uint8_t* scales = nullptr;
  uint8_t* scales_tc = nullptr;
  uint8_t* meta = nullptr;       // sparse A: pair metadata [rows][K/16]
  void free() {
    cudaFree(packed);
    cudaFree(scales);
    cudaFree(scales_tc);
    cudaFree(meta);
  }
};

// Sparse mode: block 32 scales for A and B (the sparse MMA's block); sparse_a: prune A with a
// seeded pair pattern and compress it (the dequantised copy keeps the pruned dense values).
Operand make_operand(int rows, int K, uint64_t seed, bool normal, float* keep_dequant,
                     bool sparse_mode = false, bool sparse_a = false) {
  Operand o;
  float* x = nullptr;
  CK(cudaMalloc(&x, sizeof(float) * size_t(rows) * K));
  std::string err;
  bool ok = normal ? nvfp4b200::fill_normal(x, size_t(rows) * K, seed, 0, &err)
                   : nvfp4b200::fill_uniform(x, size_t(rows) * K, seed, 0, &err);
  const int block = sparse_mode ? 32 : 16;
  if (ok && sparse_a) {
    CK(cudaMalloc(&o.meta, size_t(rows) * K / 16));
    ok = nvfp4b200::sparse_meta(rows, K, 0x24, o.meta, 0, &err) &&
         nvfp4b200::sparse_prune(x, rows, K, o.meta, 0, &err);
  }
  CK(cudaMalloc(&o.packed, size_t(rows) * K / 2));
  CK(cudaMalloc(&o.scales, size_t(rows) * K / block));
  CK(cudaMalloc(&o.scales_tc, nvfp4b200::sf_tcgen05_bytes(rows, block == 16 ? K : K / 2)));
  ok = ok && nvfp4b200::quantize_block(x, rows, K, 1.0f, block, o.packed, o.scales, o.scales_tc, 0, &err);
  if (ok && keep_dequant)
    ok = nvfp4b200::dequantize_block(o.packed, o.scales, rows, K, 1.0f, block, keep_dequant, 0, &err);
  if (ok && sparse_a) {
    uint8_t* vals = nullptr;
    CK(cudaMalloc(&vals, size_t(rows) * K / 4));
    ok = nvfp4b200::sparse_compress(o.packed, rows, K, o.meta, vals, 0, &err);
    CK(cudaDeviceSynchronize());
    cudaFree(o.packed);
    o.packed = vals;
  }
  if (!ok) {
    std::fprintf(stderr, "operand set-up failed: %s\n", err.c_str());
    std::exit(1);
  }
  CK(cudaFree(x));
  return o;
}

BenchResult run_bench(KernelKind kind, const GemmProblem& prob, const Dev& dev, const Config& cfg) {
  BenchResult r;
  r.problem = prob;
  r.kernel = kind;
  const int M = prob.m, N = prob.n, K = prob.k;
  float *adq = nullptr, *bdq = nullptr;
  if (cfg.validate) {
    CK(cudaMalloc(&adq, sizeof(float) * size_t(M) * K));
    CK(cudaMalloc(&bdq, sizeof(float) * size_t(N) * K));
  }
  const bool sparse = prob.mode == GemmMode::Sparse;
  Operand A = make_operand(M, K, cfg.seed, cfg.normal, adq, sparse, sparse);
  Operand B = make_operand(N, K, cfg.seed ^ 0xABCDEF, cfg.normal, bdq, sparse);  // src/bench.cu:29-30
  void* c = nullptr;
  const size_t esize = cfg.bf16 ? 2 : 4;
  CK(cudaMalloc(&c, esize * size_t(M) * N));

  Nvfp4DeviceOperands op;
  op.a_packed = A.packed;
  op.a_scales = cfg.tcgen05_sf ? A.scales_tc : A.scales;
  op.b_packed = B.packed;
  op.b_scales = cfg.tcgen05_sf ? B.scales_tc : B.scales;
  op.M = M;
  op.N = N;
  op.K = K;
  op.mode = prob.mode;
  op.a_meta = A.meta;
  op.sf_layout = cfg.tcgen05_sf ? SfLayout::Tcgen05 : SfLayout::Canonical;
  op.out_dtype = cfg.bf16 ? OutDType::BF16 : OutDType::F32;
  op.d = c;
  op.c = cfg.bf16 ? nullptr : static_cast<float*>(c);
  op.cta_group = cfg.cta_group;
  op.tile_n = cfg.tile_n;

  cudaStream_t s;
  CK(cudaStreamCreate(&s));
  std::string err;
  bool ok = true;
  for (int i = 0; i < std::max(1, cfg.warmup) && ok; ++i) ok = launch_gemm(kind, op, s, &err);
  if (!ok) {
    r.ok = false;
    r.note = err;
  } else {
    CK(cudaStreamSynchronize(s));
    cudaEvent_t e0, e1;
    CK(cudaEventCreate(&e0));
    CK(cudaEventCreate(&e1));
    std::vector<double> ms;
    for (int i = 0; i < cfg.iters; ++i) {  // src/bench.cu:90-98
      CK(cudaEventRecord(e0, s));
      launch_gemm(kind, op, s, &err);
      CK(cudaEventRecord(e1, s));
      CK(cudaEventSynchronize(e1));
      float t = 0;
      CK(cudaEventElapsedTime(&t, e0, e1));
      ms.push_back(t);
    }
    std::sort(ms.begin(), ms.end());
    r.median_ms = ms[ms.size() / 2];
    r.min_ms = ms.front();
    r.tflops = gemm_flops(prob) / (r.median_ms * 1e-3) / 1e12;
    r.peak_tflops = gemm_flops(prob) / (r.min_ms * 1e-3) / 1e12;
    if (dev.peak_tflops > 0) r.pct_dense_peak = 100.0 * r.peak_tflops / dev.peak_tflops;
    r.algorithmic_bytes = sparse ? double(M) * K / 4 + double(M) * K / 16 + double(M) * K / 32 +
                                       double(N) * K / 2 + double(N) * K / 32 + double(M) * N * esize
                                 : double(M) * K / 2 + double(M) * K / 16 + double(N) * K / 2 +
                                       double(N) * K / 16 + double(M) * N * esize;
    r.gbs = r.algorithmic_bytes / (r.min_ms * 1e-3) / 1e9;
    uint32_t* ew = nvfp4b200::device_error_word(&err);
    uint32_t word = 0;
    if (ew) CK(cudaMemcpy(&word, ew, 4, cudaMemcpyDeviceToHost));
    r.ok = word == 0;
    if (!r.ok) r.note = "device error word set (bounded wait timed out)";
    CK(cudaEventDestroy(e0));
    CK(cudaEventDestroy(e1));
  }

  if (r.ok && cfg.validate) {
    float* ref = nullptr;
    CK(cudaMalloc(&ref, sizeof(float) * size_t(M) * N));
    if (!nvfp4b200::naive_gemm_nt(adq, bdq, M, N, K, ref, s, &err)) {
      r.note = err;
    } else {
      CK(cudaStreamSynchronize(s));
      std::vector<float> hr(size_t(M) * N);
      std::vector<float> hg(size_t(M) * N);
      CK(cudaMemcpy(hr.data(), ref, sizeof(float) * hr.size(), cudaMemcpyDeviceToHost));
      if (cfg.bf16) {
        std::vector<uint16_t> hb(hg.size());
        CK(cudaMemcpy(hb.data(), c, 2 * hb.size(), cudaMemcpyDeviceToHost));
        for (size_t i = 0; i < hb.size(); ++i) {
          uint32_t u = uint32_t(hb[i]) << 16;
          std::memcpy(&hg[i], &u, 4);
        }
      } else {
        CK(cudaMemcpy(hg.data(), c, sizeof(float) * hg.size(), cudaMemcpyDeviceToHost));
      }
      double max_err = 0, cinf = 0, max_rel = 0;
      for (size_t i = 0; i < hg.size(); ++i) {
        const double e = std::fabs(double(hg[i]) - hr[i]);
        max_err = std::max(max_err, std::isnan(e) ? 1e300 : e);
        cinf = std::max(cinf, std::fabs(double(hr[i])));
        max_rel = std::max(max_rel, e / std::max(1e-6, std::fabs(double(hr[i]))));  // src/reference.cu:45-56
      }
      r.validated = true;
      r.max_rel_err = max_rel;
      r.max_abs_err_over_cinf = max_err / std::max(cinf, 1e-30);
      // BF16 output: allow the final rounding (half a BF16 ulp of max|C|).
      r.valid_pass = r.max_abs_err_over_cinf <= cfg.tol + (cfg.bf16 ? std::ldexp(1.0, -8) : 0.0);
    }
    cudaFree(ref);
  }
  CK(cudaStreamDestroy(s));
  A.free();
  B.free();
  cudaFree(c);
  cudaFree(adq);
  cudaFree(bdq);
  return r;
}

void print_header() {
  std::printf("%-7s %-20s %-6s %9s %10s %10s %8s %9s  %s\n", "kernel", "MxNxK", "mode", "best_ms",
              "peakTFLOPS", "sustTFLOPS", "%ladder", "GB/s", "validation");
  std::printf("%s\n", std::string(110, '-').c_str());
}

void print_result(const BenchResult& r) {
  char dims[64];
  std::snprintf(dims, sizeof(dims), "%dx%dx%d", r.problem.m, r.problem.n, r.problem.k);
  if (!r.ok) {
    std::printf("%-7s %-20s %-6s   --- not run: %s\n", to_string(r.kernel), dims,
                to_string(r.problem.mode), r.note.c_str());
    return;
  }
  char val[96] = "";
  if (r.validated)
    std::snprintf(val, sizeof(val), "%s (err/|C| %.2e, relerr %.2e)", r.valid_pass ? "PASS" : "FAIL",
                  r.max_abs_err_over_cinf, r.max_rel_err);
  std::printf("%-7s %-20s %-6s %9.4f %10.1f %10.1f %7.1f%% %9.0f  %s\n", to_string(r.kernel), dims,
              to_string(r.problem.mode), r.min_ms, r.peak_tflops, r.tflops, r.pct_dense_peak, r.gbs,
              val);
}

void write_csv(const std::string& path, const std::vector<BenchResult>& rows) {  // src/bench.cu:154-164
  std::ofstream f(path);
  f << "kernel,M,N,K,mode,median_ms,min_ms,sust_tflops,peak_tflops,pct_ladder,gbs,validated,pass,"
       "max_rel_err,err_over_cinf,note\n";
  for (const auto& r : rows)
    f << to_string(r.kernel) << ',' << r.problem.m << ',' << r.problem.n << ',' << r.problem.k << ','
      << to_string(r.problem.mode) << ',' << r.median_ms << ',' << r.min_ms << ',' << r.tflops << ','
      << r.peak_tflops << ',' << r.pct_dense_peak << ',' << r.gbs << ',' << (r.validated ? 1 : 0) << ','
      << (r.valid_pass ? 1 : 0) << ',' << r.max_rel_err << ',' << r.max_abs_err_over_cinf << ",\""
      << r.note << "\"\n";
}

void write_json(const std::string& path, const std::vector<BenchResult>& rows, const Dev& dev) {
  std::ofstream f(path);  // src/bench.cu:166-187
  f << "{\n  \"device\": {\"name\": \"" << dev.name << "\", \"sm_count\": " << dev.sms
    << ", \"measured_fp4_dense_tflops\": " << dev.peak_tflops << "},\n  \"results\": [\n";
  for (size_t i = 0; i < rows.size(); ++i) {
    const auto& r = rows[i];
    f << "    {\"kernel\": \"" << to_string(r.kernel) << "\", \"M\": " << r.problem.m
      << ", \"N\": " << r.problem.n << ", \"K\": " << r.problem.k << ", \"mode\": \""
      << to_string(r.problem.mode) << "\", \"median_ms\": " << r.median_ms << ", \"min_ms\": " << r.min_ms
      << ", \"sust_tflops\": " << r.tflops << ", \"peak_tflops\": " << r.peak_tflops
      << ", \"pct_ladder\": " << r.pct_dense_peak << ", \"gbs\": " << r.gbs
      << ", \"ok\": " << (r.ok ? "true" : "false") << ", \"validated\": " << (r.validated ? "true" : "false")
      << ", \"pass\": " << (r.valid_pass ? "true" : "false") << ", \"max_rel_err\": " << r.max_rel_err
      << ", \"err_over_cinf\": " << r.max_abs_err_over_cinf << "}" << (i + 1 < rows.size() ? ",\n" : "\n");
  }
  f << "  ]\n}\n";
}

// The tcgen05 FP4 ladder: zero operands (the issue-rate ceiling at full clock), then random
// E2M1 operands timed alone (burst) and back to back for about a second (sustained, under the
// power cap), each with the SM clock it ran at. Returns the random-data burst figure of the
// one-SM N=256 rung, the roof a GEMM on real operands timed alone is held to.
double run_ladder(const Dev& dev, bool print) {
  std::string err;
  double roof = 0;
  struct Rung { int n, cg; uint32_t seed; int sustained; int sparse; const char* what; };
  const Rung rungs[] = {{128, 1, 0u, 0, 0, "zero data, burst"},  {256, 1, 0u, 0, 0, "zero data, burst"},
                        {256, 2, 0u, 0, 0, "zero data, burst"},  {256, 1, 0x5EEDu, 0, 0, "random data, burst"},
                        {256, 2, 0x5EEDu, 0, 0, "random data, burst"},
                        {256, 1, 0x5EEDu, 1, 0, "random data, sustained ~1 s"},
                        {256, 2, 0x5EEDu, 1, 0, "random data, sustained ~1 s"},
                        {128, 1, 0x5EEDu, 0, 1, "sparse .sp (K 128), random data, burst"},
                        {256, 1, 0x5EEDu, 0, 1, "sparse .sp (K 128), random data, burst"}};
  for (const Rung& r : rungs) {
    const int units = r.cg == 2 ? dev.sms / 2 : dev.sms;
    const nvfp4b200::PeakOptions o{r.n, r.cg, units, 4096, r.sustained ? 3000 : 10, r.seed, r.sustained, r.sparse};
    double tf = 0, mhz = 0;
    if (!nvfp4b200::peak_ladder_ex(o, &tf, &mhz, 0, &err)) {
      std::printf("peak ladder failed: %s\n", err.c_str());
      return roof;
    }
    if (print)
      std::printf("tcgen05 kind::mxf4nvf4 block_scale %s M%d x N%d x K%d, %d %s, %s: %8.1f TFLOPS at %.0f MHz\n",
                  r.cg == 2 ? "cta_group::2" : "cta_group::1", r.cg == 2 ? 256 : 128, r.n,
                  r.sparse ? 128 : 64, units,
                  r.cg == 2 ? "SM pairs" : "CTAs", r.what, tf, mhz);
    if (r.cg == 1 && r.n == 256 && r.seed && !r.sustained) roof = tf;
  }
  return roof;
}

void run_bandwidth() {
  const size_t bytes = size_t(2) << 30;
  void *a = nullptr, *b = nullptr, *c = nullptr;
  CK(cudaMalloc(&a, bytes));
  CK(cudaMalloc(&b, bytes));
  CK(cudaMalloc(&c, bytes));
  CK(cudaMemset(a, 1, bytes));
  CK(cudaMemset(b, 2, bytes));
  const char* names[3] = {"copy (read+write)", "read-only", "triad (2 reads + 1 write)"};
  for (int kind = 0; kind < 3; ++kind) {
    double gbs = 0;
    std::string err;
    if (nvfp4b200::measure_bandwidth(kind, a, c, kind == 2 ? b : nullptr, bytes, 20, &gbs, 0, &err))
      std::printf("HBM %-26s %8.0f GB/s\n", names[kind], gbs);
    else
      std::printf("HBM %-26s failed: %s\n", names[kind], err.c_str());
  }
  cudaFree(a);
  cudaFree(b);
  cudaFree(c);
}

}  // namespace

// SM clocks through NVML, reading only (the reference's query_clocks_nvml,
// src/device_probe.cu:13-32). libnvidia-ml is opened at run time, so the harness neither links
// nor needs it; the device is matched by PCI bus id, since NVML and CUDA may number devices
// differently. Returns false when NVML or a query is unavailable.
static bool nvml_sm_clocks(int cuda_device, int& max_mhz, int& cur_mhz) {
  void* h = dlopen("libnvidia-ml.so.1", RTLD_LAZY | RTLD_LOCAL);
  if (!h) return false;
  using InitFn = int (*)();
  using ByPciFn = int (*)(const char*, void**);
  using ClockFn = int (*)(void*, int, unsigned int*);
  auto init = reinterpret_cast<InitFn>(dlsym(h, "nvmlInit_v2"));
  auto shutdown = reinterpret_cast<InitFn>(dlsym(h, "nvmlShutdown"));
  auto by_pci = reinterpret_cast<ByPciFn>(dlsym(h, "nvmlDeviceGetHandleByPciBusId_v2"));
  auto max_clock = reinterpret_cast<ClockFn>(dlsym(h, "nvmlDeviceGetMaxClockInfo"));
  auto clock = reinterpret_cast<ClockFn>(dlsym(h, "nvmlDeviceGetClockInfo"));
  bool ok = false;
  char bus[32] = {0};
  if (init && shutdown && by_pci && max_clock && clock &&
      cudaDeviceGetPCIBusId(bus, sizeof(bus), cuda_device) == cudaSuccess && init() == 0) {
    void* dev = nullptr;
    constexpr int kClockSm = 1;  // NVML_CLOCK_SM
    unsigned int mx = 0, cur = 0;
    if (by_pci(bus, &dev) == 0) {
      const bool a = max_clock(dev, kClockSm, &mx) == 0;
      const bool b = clock(dev, kClockSm, &cur) == 0;
      if (a) max_mhz = static_cast<int>(mx);
      if (b) cur_mhz = static_cast<int>(cur);
      ok = a || b;
    }
    shutdown();
  }
  dlclose(h);
  return ok;
}

int main(int argc, char** argv) {
  std::string kernel_sel = "b200", mode_sel = "dense", csv_path, json_path;
  int m = 4096, n = 14336, k = 4096, device = 0;
  bool sweep = false, do_bw = false, do_peak = false;
  Config cfg;
  for (int i = 1; i < argc; ++i) {
    const char* a = argv[i];
    auto next = [&](const char* name) -> const char* {
      if (i + 1 >= argc) {
        std::fprintf(stderr, "missing value for %s\n", name);
        std::exit(2);
      }
      return argv[++i];
    };
    if (eq(a, "-h") || eq(a, "--help")) { usage(argv[0]); return 0; }
    else if (eq(a, "--kernel")) kernel_sel = next(a);
    else if (eq(a, "--mode")) mode_sel = next(a);
    else if (eq(a, "--m")) m = std::atoi(next(a));
    else if (eq(a, "--n")) n = std::atoi(next(a));
    else if (eq(a, "--k")) k = std::atoi(next(a));
    else if (eq(a, "--sweep")) sweep = true;
    else if (eq(a, "--iters")) cfg.iters = std::atoi(next(a));
    else if (eq(a, "--warmup")) cfg.warmup = std::atoi(next(a));
    else if (eq(a, "--validate")) cfg.validate = true;
    else if (eq(a, "--tol")) cfg.tol = std::atof(next(a));
    else if (eq(a, "--dist")) cfg.normal = !eq(next(a), "uniform");
    else if (eq(a, "--out")) cfg.bf16 = eq(next(a), "bf16");
    else if (eq(a, "--sf")) cfg.tcgen05_sf = !eq(next(a), "canonical");
    else if (eq(a, "--cta-group")) cfg.cta_group = std::atoi(next(a));
    else if (eq(a, "--tile-n")) cfg.tile_n = std::atoi(next(a));
    else if (eq(a, "--peak")) do_peak = true;
    else if (eq(a, "--bandwidth")) do_bw = true;
    else if (eq(a, "--device")) device = std::atoi(next(a));
    else if (eq(a, "--csv")) csv_path = next(a);
    else if (eq(a, "--json")) json_path = next(a);
    else { std::fprintf(stderr, "unknown arg: %s\n", a); usage(argv[0]); return 2; }
  }
  CK(cudaSetDevice(device));
  cudaDeviceProp prop;
  CK(cudaGetDeviceProperties(&prop, device));
  Dev dev;
  dev.id = device;
  dev.name = prop.name;
  dev.sms = prop.multiProcessorCount;
  std::printf("Device %d: %s, sm_%d%d, %d SMs, %.1f GB, L2 %d MB\n\n", device, prop.name, prop.major,
              prop.minor, prop.multiProcessorCount, prop.totalGlobalMem / 1e9, prop.l2CacheSize >> 20);
  {
    int max_mhz = 0, cur_mhz = 0;
    if (nvml_sm_clocks(device, max_mhz, cur_mhz))
      std::printf("SM clock (NVML): max %d MHz, current %d MHz\n\n", max_mhz, cur_mhz);
    else
      std::printf("SM clock (NVML): unavailable\n\n");
  }
  if (prop.major != 10) std::printf("warning: this engine targets sm_100 (B200)\n");
  if (do_bw) { run_bandwidth(); std::printf("\n"); }
  if (do_peak) { run_ladder(dev, true); return 0; }
  dev.peak_tflops = run_ladder(dev, false);

  std::vector<KernelKind> kernels;
  auto want = [&](const char* s) { return kernel_sel == "all" || kernel_sel == s; };
  if (want("stub")) kernels.push_back(KernelKind::Stub);
  if (want("cutlass")) kernels.push_back(KernelKind::Cutlass);
  if (want("custom")) kernels.push_back(KernelKind::Custom);
  if (want("b200")) kernels.push_back(KernelKind::B200);
  if (kernels.empty()) { std::fprintf(stderr, "no kernel selected\n"); return 2; }
  std::vector<GemmMode> modes;
  if (mode_sel == "dense" || mode_sel == "both") modes.push_back(GemmMode::Dense);
  if (mode_sel == "sparse" || mode_sel == "both") modes.push_back(GemmMode::Sparse);
  std::vector<GemmProblem> sizes;
  if (sweep) {  // src/main.cu:105-116 plus the BASELINE configurations
    for (auto t : {std::vector<int>{4096, 14336, 4096}, {4096, 28672, 4096}, {6144, 6144, 6144},
                   {2048, 2048, 2048}, {4096, 4096, 4096}, {8192, 8192, 8192}, {12288, 12288, 12288},
                   {16384, 16384, 16384}, {1024, 1024, 1024}, {16, 14336, 4096}, {64, 14336, 4096},
                   {128, 14336, 4096}, {16, 4096, 14336}, {64, 4096, 14336}, {128, 4096, 14336}})
      sizes.push_back(GemmProblem{t[0], t[1], t[2], GemmMode::Dense});
  } else {
    sizes.push_back(GemmProblem{m, n, k, GemmMode::Dense});
  }
  print_header();
  std::vector<BenchResult> rows;
  for (auto sz : sizes)
    for (auto mode : modes)
      for (auto kk : kernels) {
        GemmProblem p = sz;
        p.mode = mode;
        BenchResult r = run_bench(kk, p, dev, cfg);
        print_result(r);
        rows.push_back(r);
      }
  if (!csv_path.empty()) { write_csv(csv_path, rows); std::printf("\nWrote %s\n", csv_path.c_str()); }
  if (!json_path.empty()) { write_json(json_path, rows, dev); std::printf("Wrote %s\n", json_path.c_str()); }
  bool all_pass = true;
  for (const auto& r : rows)
    if (r.validated && !r.valid_pass) all_pass = false;
  return all_pass ? 0 : 1;
}
