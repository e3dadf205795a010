/* nvfp4_oracle.c - CPU restatement of the reference's NVFP4 codecs and FP32 GEMM oracle.
 *
 * TEST INFRASTRUCTURE ONLY: the checker for the CUDA product path, never the product.
 * Build: oracle/Makefile (gcc -O2 -ffp-contract=off, pthreads; no fast-math, so every float
 * operation below is one IEEE-754 single-precision operation, as in the reference's
 * host code compiled for x86-64).
 *
 * Each function cites the reference line it restates (paths inside the reference project).
 */
#include "nvfp4_oracle.h"

#include <math.h>
#include <pthread.h>
#include <string.h>
#include <unistd.h>

/* Minimal parallel-for over [0, n) in contiguous chunks on pthreads (the image ships no
 * OpenMP runtime). threads <= 0 means one thread per online host core. */
typedef void (*range_fn)(void* ctx, long lo, long hi);
typedef struct { range_fn fn; void* ctx; long lo, hi; } range_job;
static void* range_tramp(void* p) {
  range_job* j = (range_job*)p;
  j->fn(j->ctx, j->lo, j->hi);
  return NULL;
}
int orc_default_threads(void) {
  long n = sysconf(_SC_NPROCESSORS_ONLN);
  return n > 0 ? (int)n : 1;
}
static void parallel_range(long n, int threads, range_fn fn, void* ctx) {
  if (threads <= 0) threads = orc_default_threads();
  if (threads > 256) threads = 256;
  if ((long)threads > n) threads = (int)(n > 0 ? n : 1);
  if (threads <= 1) { fn(ctx, 0, n); return; }
  pthread_t tid[256];
  range_job job[256];
  int live[256];
  long chunk = (n + threads - 1) / threads;
  for (int t = 0; t < threads; ++t) {
    long lo = (long)t * chunk, hi = lo + chunk < n ? lo + chunk : n;
    live[t] = 0;
    if (lo >= hi) continue;
    job[t].fn = fn; job[t].ctx = ctx; job[t].lo = lo; job[t].hi = hi;
    if (pthread_create(&tid[t], NULL, range_tramp, &job[t]) == 0) live[t] = 1;
    else fn(ctx, lo, hi);
  }
  for (int t = 0; t < threads; ++t)
    if (live[t]) pthread_join(tid[t], NULL);
}

/* src/nvfp4.cu:10 - positive E2M1 magnitudes indexed by (exp<<1 | mant) */
static const float kMag[8] = {0.0f, 0.5f, 1.0f, 1.5f, 2.0f, 3.0f, 4.0f, 6.0f};

/* src/nvfp4.cu:13-16 */
float orc_e2m1_decode(uint8_t code) {
  float m = kMag[code & 0x7];
  return (code & 0x8) ? -m : m;
}

/* src/nvfp4.cu:18-29. The strict '<' keeps the first (smaller) magnitude on a tie, and a
 * NaN never compares smaller, so NaN (and +-inf, whose errors are all inf) map to
 * magnitude code 0. */
uint8_t orc_e2m1_quantize(float x) {
  uint8_t sign = (x < 0.0f) ? 0x8 : 0x0;
  float a = fabsf(x);
  int best = 0;
  float best_err = fabsf(a - kMag[0]);
  for (int i = 1; i < 8; ++i) {
    float e = fabsf(a - kMag[i]);
    if (e < best_err) { best_err = e; best = i; }
  }
  return (uint8_t)(sign | (uint8_t)best);
}

/* src/nvfp4.cu:34-45. ldexpf of a small exact value is exact, so this equals std::ldexp. */
float orc_e4m3_decode(uint8_t code) {
  int sign = (code >> 7) & 1;
  int e = (code >> 3) & 0xF;
  int m = code & 0x7;
  float v = (e == 0) ? ldexpf((float)m / 8.0f, 1 - 7) : ldexpf(1.0f + (float)m / 8.0f, e - 7);
  return sign ? -v : v;
}

/* src/nvfp4.cu:47-59. x <= 0 -> 0; min(x, 448) keeps NaN (std::min(a,b) returns a unless
 * b < a), and a NaN error never wins, so NaN -> code 0. */
uint8_t orc_e4m3_encode(float x) {
  if (x <= 0.0f) return 0;
  if (448.0f < x) x = 448.0f;
  uint8_t best = 0;
  float best_err = 1e30f;
  for (int c = 0; c < 128; ++c) {
    float v = orc_e4m3_decode((uint8_t)c);
    float e = fabsf(v - x);
    if (e < best_err) { best_err = e; best = (uint8_t)c; }
  }
  return best;
}

/* src/nvfp4.cu:62-97. amax uses std::max(amax, |x|), which ignores NaN. */
typedef struct { const float* src; int cols; float g; uint8_t* packed; uint8_t* scales; int blk; } quant_ctx;
static void quant_rows(void* p, long r0, long r1) {
  const quant_ctx* q = (const quant_ctx*)p;
  const float* src = q->src;
  const int blk = q->blk, cols = q->cols, nb = cols / blk;
  const float global_scale = q->g;
  uint8_t* packed = q->packed;
  uint8_t* scales = q->scales;
  for (long r = r0; r < r1; ++r) {
    for (int b = 0; b < nb; ++b) {
      const float* x = src + (size_t)r * cols + (size_t)b * blk;
      float amax = 0.0f;
      for (int j = 0; j < blk; ++j) {
        float a = fabsf(x[j]);
        if (amax < a) amax = a;
      }
      float scale = (amax > 0.0f) ? (amax / 6.0f) / global_scale : 1.0f;
      uint8_t sc = orc_e4m3_encode(scale);
      float dec = orc_e4m3_decode(sc) * global_scale;
      if (dec <= 0.0f) dec = 1.0f;
      scales[(size_t)r * nb + b] = sc;
      for (int j = 0; j < blk; ++j) {
        size_t c = (size_t)b * blk + (size_t)j;
        uint8_t code = orc_e2m1_quantize(x[j] / dec);
        size_t bi = ((size_t)r * cols + c) / 2;
        if ((c & 1) == 0) packed[bi] = (uint8_t)((packed[bi] & 0xF0) | (code & 0x0F));
        else packed[bi] = (uint8_t)((packed[bi] & 0x0F) | (uint8_t)((code & 0x0F) << 4));
      }
    }
  }
}

void orc_quantize(const float* src, int rows, int cols, float global_scale,
                  uint8_t* packed, uint8_t* scales) {
  orc_quantize_block(src, rows, cols, global_scale, 16, packed, scales);
}

/* The same algorithm with `block` contiguous elements per scale (16 = src/nvfp4.cu; 32 = the
 * block the sparse tensor-core MMA applies, one scale per 32 logical K elements). */
void orc_quantize_block(const float* src, int rows, int cols, float global_scale, int block,
                        uint8_t* packed, uint8_t* scales) {
  quant_ctx q = {src, cols, global_scale, packed, scales, block};
  memset(packed, 0, (size_t)rows * (size_t)(cols / 2));
  parallel_range(rows, 0, quant_rows, &q);
}

/* src/nvfp4.cu:99-112 */
typedef struct { const uint8_t* packed; const uint8_t* scales; int cols; float g; float* out; int blk; } dq_ctx;
static void dq_rows(void* p, long r0, long r1) {
  const dq_ctx* q = (const dq_ctx*)p;
  const uint8_t* packed = q->packed;
  const uint8_t* scales = q->scales;
  const int blk = q->blk, cols = q->cols, nb = cols / blk;
  const float global_scale = q->g;
  float* out = q->out;
  for (long r = r0; r < r1; ++r) {
    for (int c = 0; c < cols; ++c) {
      size_t bi = ((size_t)r * cols + c) / 2;
      uint8_t byte = packed[bi];
      uint8_t code = (c & 1) ? (uint8_t)(byte >> 4) : (uint8_t)(byte & 0x0F);
      float s = orc_e4m3_decode(scales[(size_t)r * nb + c / blk]) * global_scale;
      out[(size_t)r * cols + c] = orc_e2m1_decode(code) * s;
    }
  }
}

void orc_dequantize(const uint8_t* packed, const uint8_t* scales, int rows, int cols,
                    float global_scale, float* out) {
  orc_dequantize_block(packed, scales, rows, cols, global_scale, 16, out);
}

void orc_dequantize_block(const uint8_t* packed, const uint8_t* scales, int rows, int cols,
                          float global_scale, int block, float* out) {
  dq_ctx q = {packed, scales, cols, global_scale, out, block};
  parallel_range(rows, 0, dq_rows, &q);
}

static inline uint64_t splitmix_mix(uint64_t z) {
  z = (z ^ (z >> 30)) * 0xBF58476D1CE4E5B9ull;
  z = (z ^ (z >> 27)) * 0x94D049BB133111EBull;
  return z ^ (z >> 31);
}

/* src/nvfp4.cu:115-129. The state after i+1 steps is seed + (i+1)*golden, so element i is a
 * pure function of its index (the GPU generator relies on the same fact). */
void orc_make_uniform(int rows, int cols, uint64_t seed, float* out) {
  const uint64_t g = 0x9E3779B97F4A7C15ull;
  uint64_t x0 = seed ? seed : g;
  size_t n = (size_t)rows * (size_t)cols;
  for (size_t i = 0; i < n; ++i) {
    uint64_t z = splitmix_mix(x0 + (uint64_t)(i + 1) * g);
    out[i] = ((float)(z >> 40) / (float)(1 << 24)) * 2.0f - 1.0f;
  }
}

/* src/reference.cu:9-17. B is N x K here (the engine's layout), so the k loop reads both
 * operands contiguously; the summation order (k ascending, one fp32 accumulator) is the
 * reference's. */
static void gemm_row(const float* a, const float* B, int N, int K, float* c) {
  for (int n = 0; n < N; ++n) {
    const float* b = B + (size_t)n * K;
    float acc = 0.0f;
    for (int k = 0; k < K; ++k) acc += a[k] * b[k];
    c[n] = acc;
  }
}

typedef struct { const float* A; const float* B; int N, K; const int* rows; float* C; } gemm_ctx;
static void gemm_rows(void* p, long i0, long i1) {
  const gemm_ctx* g = (const gemm_ctx*)p;
  for (long i = i0; i < i1; ++i) {
    long m = g->rows ? g->rows[i] : i;
    gemm_row(g->A + (size_t)m * g->K, g->B, g->N, g->K, g->C + (size_t)i * g->N);
  }
}

void orc_gemm_nt(const float* A, const float* B, int M, int N, int K, float* C, int threads) {
  gemm_ctx g = {A, B, N, K, NULL, C};
  parallel_range(M, threads, gemm_rows, &g);
}

void orc_gemm_nt_rows(const float* A, const float* B, int M, int N, int K,
                      const int* rows, int nrows, float* C_rows, int threads) {
  (void)M;
  gemm_ctx g = {A, B, N, K, rows, C_rows};
  parallel_range(nrows, threads, gemm_rows, &g);
}

/* src/reference.cu:45-56 */
double orc_max_rel_error(const float* got, const float* ref, size_t n) {
  double worst = 0.0;
  for (size_t i = 0; i < n; ++i) {
    double r = ref[i], g = got[i];
    double d = fabs(r);
    if (d < 1e-6) d = 1e-6;
    double e = fabs(g - r) / d;
    if (e > worst) worst = e;
  }
  return worst;
}

void orc_max_abs_error(const float* got, const float* ref, size_t n, double* max_err,
                       double* max_ref) {
  double me = 0.0, mr = 0.0;
  for (size_t i = 0; i < n; ++i) {
    double e = fabs((double)got[i] - (double)ref[i]);
    if (e > me || e != e) me = (e != e) ? INFINITY : e;
    double r = fabs((double)ref[i]);
    if (r > mr) mr = r;
  }
  *max_err = me;
  *max_ref = mr;
}

size_t orc_sf_tcgen05_bytes(int rows, int K) {
  size_t rb = ((size_t)rows + 127) / 128;
  size_t kb = ((size_t)K + 63) / 64;
  return rb * kb * 512;
}

void orc_sf_to_tcgen05(const uint8_t* scales, int rows, int K, uint8_t* out) {
  const int ns = K / 16;
  const size_t kb = ((size_t)K + 63) / 64;
  memset(out, 0, orc_sf_tcgen05_bytes(rows, K));
  for (int r = 0; r < rows; ++r)
    for (int s = 0; s < ns; ++s) {
      size_t atom = ((size_t)r / 128) * kb + (size_t)s / 4;
      size_t off = atom * 512 + (size_t)(r % 32) * 16 + (size_t)((r / 32) % 4) * 4 + (size_t)(s % 4);
      out[off] = scales[(size_t)r * ns + s];
    }
}

/* The 6 ways to keep 2 of 4: first and second kept index. */
static const uint8_t kPairLo[6] = {0, 0, 0, 1, 1, 2};
static const uint8_t kPairHi[6] = {1, 2, 3, 2, 3, 3};


/* Pair-wise 2:4 sparsity of A (the pattern the tcgen05 .sp kind::mxf4nvf4 MMA executes,
 * measured on B200): each group of 8 consecutive K elements of a row is 4 element pairs, of
 * which 2 are kept. Group i = row*K/8 + g keeps the pair combination
 * splitmix64(seed + (i+1)*golden) % 6 of {01, 02, 03, 12, 13, 23}; its metadata nibble is
 * first_pair | second_pair << 2, two groups per byte (even group in the low nibble). */
void orc_sparse_meta(int rows, int K, uint64_t seed, uint8_t* meta) {
  const uint64_t g = 0x9E3779B97F4A7C15ull;
  const size_t n = (size_t)rows * (size_t)(K / 8);
  memset(meta, 0, n / 2);
  for (size_t i = 0; i < n; ++i) {
    const unsigned p = (unsigned)(splitmix_mix(seed + (uint64_t)(i + 1) * g) % 6);
    const uint8_t nib = (uint8_t)(kPairLo[p] | (kPairHi[p] << 2));
    meta[i / 2] |= (uint8_t)(nib << (4 * (i & 1)));
  }
}

static inline uint8_t meta_nibble(const uint8_t* meta, size_t i) { return (uint8_t)((meta[i / 2] >> (4 * (i & 1))) & 0xF); }

/* Zero the elements of the two dropped pairs of every group (fp32, in place). */
void orc_sparse_prune(float* a, int rows, int K, const uint8_t* meta) {
  const size_t n = (size_t)rows * (size_t)(K / 8);
  for (size_t i = 0; i < n; ++i) {
    const uint8_t nib = meta_nibble(meta, i);
    const int p0 = nib & 3, p1 = (nib >> 2) & 3;
    for (int pr = 0; pr < 4; ++pr)
      if (pr != p0 && pr != p1) a[i * 8 + 2 * pr] = a[i * 8 + 2 * pr + 1] = 0.0f;
  }
}

/* Packed [rows][K/2] -> compressed [rows][K/4]: one pair is one byte, so group i keeps bytes
 * 4i + first and 4i + second, in that order. */
void orc_sparse_compress(const uint8_t* packed, int rows, int K, const uint8_t* meta, uint8_t* values) {
  const size_t n = (size_t)rows * (size_t)(K / 8);
  for (size_t i = 0; i < n; ++i) {
    const uint8_t nib = meta_nibble(meta, i);
    values[2 * i] = packed[4 * i + (nib & 3)];
    values[2 * i + 1] = packed[4 * i + ((nib >> 2) & 3)];
  }
}
