/* nvfp4_b200.h - C ABI of the B200 NVFP4 GEMM engine (libnvfp4_b200.so).
 *
 * Plain pointers and sizes only. Every entry point returns 0 on success, or a nonzero
 * NVFP4_B200_E* code with a message copied into `err` (up to errlen bytes, may be NULL);
 * none throws or exits, and all launches are asynchronous on `stream` (a cudaStream_t; NULL
 * = legacy default stream) on the current device. Device buffers belong to the caller.
 * This is the surface a ctypes / cgo / JNI binding of the reference's hot path binds;
 * each declaration names the reference interface it replaces (paths inside the reference
 * project).
 */
#ifndef NVFP4_B200_H
#define NVFP4_B200_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

enum {
  NVFP4_B200_OK = 0,
  NVFP4_B200_EINVAL = 1,       /* bad argument (null pointer, unsupported shape or mode) */
  NVFP4_B200_ECUDA = 2,        /* a CUDA runtime/driver call failed */
  NVFP4_B200_EUNSUPPORTED = 3, /* device is not sm_100 or the feature is not built */
  NVFP4_B200_EDEVICE = 4       /* a kernel reported a bounded-wait timeout (device error word) */
};

/* GemmMode / SfLayout / OutDType values (include/gemm.h). */
enum { NVFP4_MODE_DENSE = 0, NVFP4_MODE_SPARSE24 = 1 };
enum { NVFP4_SF_CANONICAL = 0, NVFP4_SF_TCGEN05 = 1 };
enum { NVFP4_OUT_F32 = 0, NVFP4_OUT_BF16 = 1, NVFP4_OUT_NVFP4 = 2 };

/* Flat form of Nvfp4DeviceOperands (include/gemm.h; reference src/gemm.h:13-23). */
typedef struct Nvfp4GemmArgs {
  const void* a_packed; /* [M][K/2] (dense) or [M][K/4] kept values (2:4) */
  const void* a_scales; /* per sf_layout, over the logical K */
  float a_global;
  const void* b_packed; /* [N][K/2] */
  const void* b_scales;
  float b_global;
  void* c;              /* M x N row-major, element type out_dtype */
  int M, N, K;
  int mode;             /* NVFP4_MODE_* */
  int sf_layout;        /* NVFP4_SF_* */
  int out_dtype;        /* NVFP4_OUT_* */
  const void* a_meta;   /* 2:4 metadata, mode == NVFP4_MODE_SPARSE24 only */
  int cta_group;        /* 0 = heuristic, 1 or 2 */
  int tile_n;           /* 0 = heuristic, else 128 or 256 (one-SM dense tiles) */
  /* out_dtype NVFP4_OUT_NVFP4: c = packed [M][N/2] (N % 32 == 0), c_scales = its UE4M3 scales
   * in c_sf_layout (canonical [M][N/16] or tcgen05, nvfp4_b200_sf_tcgen05_bytes(M, N)),
   * quantised from alpha*acc exactly as quantize_to_nvfp4 (src/nvfp4.cu:62-97) with global
   * scale c_global: the next layer's A operand, byte-identical to quantising the FP32 output. */
  void* c_scales;
  float c_global;
  int c_sf_layout;
  int flags;            /* NVFP4_FLAG_* */
  /* Row pitch of c in elements (0 = N; FP32/BF16 output): c may be a column slice of a wider
   * row-major matrix. */
  int ldc;
  /* Fused all-gather (no reference counterpart; the reference runs on one GPU): the epilogue
   * also stores every FP32/BF16 output tile to c_peers[0 .. n_peers-1] (n_peers <= 7), each
   * addressed like c with the same pitch, typically the other ranks' output buffers mapped
   * into this process with nvfp4_b200_ipc_open. The tiles cross NVLink as they complete; when
   * this call's work has completed on `stream`, every destination holds this call's tiles.
   * Needs a 16-byte aligned c and c_peers[i] and ldc * element size a multiple of 16. */
  void* const* c_peers;
  int n_peers;
} Nvfp4GemmArgs;

/* Nvfp4GemmArgs.flags. B_STATIC: B and its scales are not written by the work enqueued just
 * before this call on the stream, so the decode kernel may start streaming the weight before
 * that work completes (e.g. while this layer's activations are being quantised). It takes
 * effect only with NVFP4_SF_TCGEN05 scales. */
enum { NVFP4_FLAG_B_STATIC = 1 };

/* Replaces launch_gemm(KernelKind::Custom, op, s, err) - src/gemm.h:31-40 and the
 * custom backend src/gemm_custom.cu:134-159 - with the tcgen05 backend. With
 * NVFP4_SF_CANONICAL the call first reorders the scales into a workspace that belongs to
 * (device, stream): calls on different streams have separate workspaces, and calls on one
 * stream are ordered by it, so concurrent canonical-scale calls do not overwrite each other's
 * scales. The workspace is allocated (cudaMalloc) on a stream's first canonical call and grown
 * when a larger problem arrives. NVFP4_FLAG_B_STATIC has no effect with canonical scales (the
 * kernel reads the reordered copy that this call itself writes); use tcgen05-layout scales for
 * it, and for callers that want no allocation at all. */
int nvfp4_b200_gemm(const Nvfp4GemmArgs* args, void* stream, char* err, size_t errlen);

/* Activation quantisation fused into the GEMM. The reference quantises both operands on the
 * host before every run (src/bench.cu:25-32, quantize_to_nvfp4 of src/nvfp4.cu:62-97); a decode
 * layer instead quantises fresh fp32 activations each step. a_src: fp32 A [M][K] (16-byte
 * aligned). args->a_packed ([M][K/2]) and args->a_scales (tcgen05 layout,
 * nvfp4_b200_sf_tcgen05_bytes(M, K)) are OUTPUTS: they receive A quantised with global scale
 * args->a_global, byte-identical to nvfp4_b200_quantize; then D = A * B^T as nvfp4_b200_gemm
 * (sf_layout must be NVFP4_SF_TCGEN05, dense). For M <= 128, K % 64 == 0, FP32/BF16 output, no
 * tile/peer options and a weight of at least half as many 128-row tiles as SMs (so that the
 * decode kernel splits no K range), this is ONE launch of the weight-streaming kernel: its
 * CTAs quantise disjoint slices of A, meet at a grid barrier (two counters in device memory,
 * bounded wait) and only then load the token tiles, while the weight stream starts at once
 * when NVFP4_FLAG_B_STATIC is set. Fused launches on one device must not overlap on the GPU
 * (they share the barrier's counters). Other shapes run the quantiser and the GEMM back to
 * back on the stream (measured faster there). */
int nvfp4_b200_gemm_quantize_a(const Nvfp4GemmArgs* args, const float* a_src, void* stream,
                               char* err, size_t errlen);

/* No counterpart in the reference. Same GEMM as nvfp4_b200_gemm with canonical scales
 * (dense mode, sf_layout must be NVFP4_SF_CANONICAL) for callers that cannot let the library
 * allocate device memory: code inside CUDA-graph capture, servers that pre-partition all GPU
 * memory into their own pool, latency-critical loops that cannot afford cudaMalloc's implicit
 * synchronisation. The scale reorder goes into a fixed 16 MiB scratch array compiled into the
 * library (held on every GPU that loads it until exit) instead of a cudaMalloc'd workspace;
 * problems whose reordered scales exceed it ((M+N)*K/16 bytes, roughly) are rejected with
 * NVFP4_B200_EINVAL. The first call on each device looks up the array's device address
 * (cudaGetSymbolAddress, with that device current): make it before any stream capture.
 * Calls share the array: calls on the same device whose work overlaps on the GPU race. */
int nvfp4_b200_gemm_noalloc(const Nvfp4GemmArgs* args, void* stream, char* err, size_t errlen);

/* Size in bytes of the scratch array nvfp4_b200_gemm_noalloc reorders scales into. No
 * counterpart in the reference. */
size_t nvfp4_b200_gemm_noalloc_scratch_bytes(void);

/* Replaces quantize_to_nvfp4 - src/nvfp4.h:40-42, src/nvfp4.cu:62-97 - on the GPU,
 * byte-identical to it. src: fp32 [rows][cols] (cols % 16 == 0). Writes packed
 * [rows][cols/2], and the scales in the canonical layout (scales, may be NULL) and/or the
 * tcgen05 layout (scales_tcgen05, may be NULL; nvfp4_b200_sf_tcgen05_bytes(rows, cols)). */
int nvfp4_b200_quantize(const float* src, int rows, int cols, float global_scale,
                        void* packed, void* scales, void* scales_tcgen05, void* stream,
                        char* err, size_t errlen);

/* Replaces dequantize_nvfp4 - src/nvfp4.h:44-45, src/nvfp4.cu:99-112 - on the GPU. */
int nvfp4_b200_dequantize(const void* packed, const void* scales, int rows, int cols,
                          float global_scale, float* out, void* stream, char* err,
                          size_t errlen);

/* quantize / dequantize with `block` (16 or 32) elements per scale. Block 16 is the
 * reference's NVFP4 codec (src/nvfp4.cu:62-112); block 32 is the same algorithm with the scale
 * block the sparse tensor-core MMA applies (one UE4M3 scale per 32 K elements of A and of B).
 * For block 32, scales are [rows][cols/32] and the tcgen05 layout takes
 * nvfp4_b200_sf_tcgen05_bytes(rows, cols / 2) bytes. */
int nvfp4_b200_quantize_ex(const float* src, int rows, int cols, float global_scale, int block,
                           void* packed, void* scales, void* scales_tcgen05, void* stream,
                           char* err, size_t errlen);
int nvfp4_b200_dequantize_ex(const void* packed, const void* scales, int rows, int cols,
                             float global_scale, int block, float* out, void* stream, char* err,
                             size_t errlen);

/* Pair-wise 2:4 structured sparsity of A (GemmMode::Sparse; the reference has no data path,
 * src/gemm_custom.cu:135-139). The tcgen05 .sp kind::mxf4nvf4 MMA keeps 2 of the 4 element
 * pairs of every group of 8 consecutive K elements. meta [rows][K/16]: one nibble per group
 * (first kept pair | second << 2; the even group in the low nibble), drawn per group i =
 * row*K/8 + g as splitmix64(seed + (i+1)*golden) % 6 over {01,02,03,12,13,23}. prune zeroes the
 * dropped pairs of an fp32 [rows][K] matrix in place; compress turns packed [rows][K/2] into
 * the kept values [rows][K/4] (one byte per kept pair, in order). K % 16 == 0. */
int nvfp4_b200_sparse_meta(int rows, int K, uint64_t seed, void* meta, void* stream, char* err,
                           size_t errlen);
int nvfp4_b200_sparse_prune(float* a, int rows, int K, const void* meta, void* stream, char* err,
                            size_t errlen);
int nvfp4_b200_sparse_compress(const void* packed, int rows, int K, const void* meta,
                               void* values, void* stream, char* err, size_t errlen);

/* Replaces make_random_matrix - src/nvfp4.h:47-48, src/nvfp4.cu:115-129 - on the GPU,
 * bit-identical (splitmix64 -> uniform [-1,1)). */
int nvfp4_b200_fill_uniform(float* out, int rows, int cols, uint64_t seed, void* stream,
                            char* err, size_t errlen);

/* N(0,1) fill (no reference counterpart; the benchmark configurations ask for it):
 * element i = Box-Muller of two splitmix64 uniforms of (seed, i). Deterministic per GPU
 * build; not bit-identical to any CPU implementation (device logf/cosf). */
int nvfp4_b200_fill_normal(float* out, int rows, int cols, uint64_t seed, void* stream,
                           char* err, size_t errlen);

/* Size in bytes of the tcgen05 scale layout for a [rows x K] operand. No reference
 * counterpart (the reference's CUTLASS backend builds its own, src/gemm_cutlass.cu:151-152). */
size_t nvfp4_b200_sf_tcgen05_bytes(int rows, int K);

/* Canonical [rows][K/16] scales -> tcgen05 layout (padding written as zero). */
int nvfp4_b200_sf_to_tcgen05(const void* scales, int rows, int K, void* out, void* stream,
                             char* err, size_t errlen);

/* Replaces measure_bandwidth_gbs - src/bench.h:24, src/bandwidth.cu:14-52 - as the HBM
 * roof. kind 0 = copy (read+write), 1 = read-only stream, 2 = triad c=a+s*b (3 arrays).
 * Uses caller-provided device buffers of `bytes` each (src, dst, src2 for triad; dst may
 * be NULL for kind 1). Returns the best GB/s over `iters` timed launches in *gbs. */
int nvfp4_b200_measure_bandwidth(int kind, const void* src, void* dst, const void* src2,
                                 size_t bytes, int iters, double* gbs, void* stream, char* err,
                                 size_t errlen);

/* Replaces run_peak_ladder - src/peak.h:8, src/peak.cu:119-156 - with a memory-free
 * tcgen05 rung: `ctas` CTAs each issue `iters` back-to-back block-scaled MMAs of shape
 * M=128 x n x K=64 (kind::mxf4nvf4, sparse = 0) into TMEM. *tflops = 2*128*n*64*ctas*iters
 * / best time over `reps` launches. */
int nvfp4_b200_peak(int n, int ctas, int iters, int reps, double* tflops, void* stream,
                    char* err, size_t errlen);

/* The same ladder with its options (src/peak.cu:119-156 has one fixed configuration):
 * cta_group 1 runs `units` CTAs of M=128 x n MMAs (n 128 or 256), cta_group 2 runs `units`
 * SM pairs of M=256 x 256 MMAs. seed 0 stages zero operands, any other value pseudo-random
 * E2M1 bytes (the data sets the power drawn and so, under the power cap, the clock).
 * sustained 0: best of `reps` single timed launches; 1: mean over `reps` back-to-back
 * launches. sparse 1 (cta_group 1): tcgen05.mma.sp rungs (128 logical K per MMA, FLOPs counted
 * on the logical K; the reference's sparse rungs, src/peak.cu:46-68,93-115). *sm_mhz (may be
 * NULL) gets the SM clock CTA 0 ran at (clock64 / globaltimer). */
int nvfp4_b200_peak_ex(int n, int cta_group, int units, int iters, int reps, uint32_t seed,
                       int sustained, int sparse, double* tflops, double* sm_mhz, void* stream,
                       char* err, size_t errlen);

/* Reads (and when clear != 0 resets) the device error word the kernels write when a
 * bounded wait times out (bit meanings in nvfp4bench_b200/csrc/ptx.cuh). Synchronises
 * the current device. Returns 0 on success with the word in *word. */
int nvfp4_b200_device_error(int clear, uint32_t* word, char* err, size_t errlen);

/* Bounded-wait self test: one CTA waits on an mbarrier that nothing completes, with a
 * limit of `limit_ns`; the kernel records NVFP4 error bit kErrTest and returns. The
 * context stays usable. Returns the device error word in *word. */
int nvfp4_b200_wait_selftest(uint64_t limit_ns, uint32_t* word, char* err, size_t errlen);

/* CUDA IPC for the fused all-gather (no reference counterpart). nvfp4_b200_ipc_handle exports
 * the device allocation holding `ptr` as NVFP4_B200_IPC_HANDLE_BYTES opaque bytes plus the
 * offset of `ptr` inside it; another process on the same node opens it with
 * nvfp4_b200_ipc_open, which returns that process's address of the same byte (opening an
 * allocation twice in one process returns the same mapping, reference-counted), and releases
 * it with nvfp4_b200_ipc_close. The exporting process keeps the allocation alive until every
 * importer has closed it. The allocation must come from cudaMalloc (PyTorch's default caching
 * allocator; not expandable segments or other virtual-memory-managed allocations, which
 * cudaIpcGetMemHandle rejects). */
enum { NVFP4_B200_IPC_HANDLE_BYTES = 64 };
int nvfp4_b200_ipc_handle(const void* ptr, void* handle, size_t* offset, char* err, size_t errlen);
int nvfp4_b200_ipc_open(const void* handle, size_t offset, void** ptr, char* err, size_t errlen);
int nvfp4_b200_ipc_close(void* ptr, char* err, size_t errlen);
/* Library version string. */
const char* nvfp4_b200_version(void);

#ifdef __cplusplus
}
#endif
#endif
