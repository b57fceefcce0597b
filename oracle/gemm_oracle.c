/*
 * CPU oracle for the f32 matmul hot path -- TEST INFRASTRUCTURE ONLY.
 *
 * This file restates, in plain C, the arithmetic of the reference CPU GEMM
 * entries of Momiru's `tensor_light` CPU provider so that the GPU kernels can
 * be checked against it. Only the test-suite, the smoke check and the CPU
 * baseline leg of the benchmark load it. The product never calls it.
 *
 * Restated reference items (paths inside the reference project):
 *   - gemm_dot_f32   src/momiru/tensor_light/execution/cpu.rs:2989-3008
 *   - gemm_axpy_f32  src/momiru/tensor_light/execution/cpu.rs:3012-3026
 *   - gemm_avx2      src/momiru/tensor_light/execution/cpu.rs:3068-3098
 *     All three produce, per output element, s = +0; for p = 0..K-1:
 *     s = s + (a[row,p] * b[p,col]) with a separately rounded f32 product and
 *     f32 sum (no FMA, increasing p). They are bit-identical, so one
 *     restatement (oracle_gemm) serves all three; oracle_gemm_avx2_restated
 *     keeps gemm_avx2's loop structure for the CPU timing baseline.
 *   - relu_f32       src/momiru/tensor_light/execution/cpu.rs:2158-2160
 *   - relu6_f32, silu_f32 (sigmoid_value)   cpu.rs:2137-2144, 2161-2168
 *   - gelu_erf_f32 (erfc_nonnegative_f64, horner)   cpu.rs:2031-2129
 *   - gelu_tanh_approx_f32                  cpu.rs:2214-2222
 *   - bias add       Elementwise Add with a trailing-axis broadcast,
 *                    src/momiru/tensor_light/execution/ir.rs:261-345
 *   - batched/broadcast matmul semantics
 *                    src/momiru/tensor_light/execution/validation.rs:2300-2398
 *   - SplitMix64, randu, randn (Box-Muller)
 *                    src/momiru/tensor_light/tensor.rs:1467-1500, 1809-1840
 *
 * Build with -ffp-contract=off and without -ffast-math (see oracle/Makefile):
 * the restatement is only bit-exact when the compiler keeps every product and
 * every sum separately rounded.
 */
#define _GNU_SOURCE
#include <math.h>
#include <pthread.h>
#include <stdint.h>
#include <stdlib.h>
#include <string.h>
#include <unistd.h>
#include <immintrin.h>

/* ------------------------------------------------------------------ RNG -- */

/* SplitMix64 step, tensor.rs:1822-1828. */
static inline uint64_t sm64_next(uint64_t *state) {
  *state += 0x9E3779B97F4A7C15ull;
  uint64_t v = *state;
  v = (v ^ (v >> 30)) * 0xBF58476D1CE4E5B9ull;
  v = (v ^ (v >> 27)) * 0x94D049BB133111EBull;
  return v ^ (v >> 31);
}

/* next_unit_f32, tensor.rs:1831-1835: high 24 bits times 2^-24, in [0,1). */
static inline float sm64_unit(uint64_t *state) {
  uint32_t bits = (uint32_t)(sm64_next(state) >> 40);
  return (float)bits * (1.0f / 16777216.0f);
}

/* Raw SplitMix64 words, for pinning the generator itself. */
void oracle_splitmix64_words(uint64_t seed, uint64_t *out, int64_t n) {
  uint64_t s = seed;
  for (int64_t i = 0; i < n; ++i) out[i] = sm64_next(&s);
}

/* randu (tensor.rs:1467-1471) mapped affinely: out = lo + (hi-lo)*u.
 * For [-1,1) this is 2u-1, which is exact in f32 for every 24-bit u. */
void oracle_randu(float *out, int64_t n, uint64_t seed, float lo, float hi) {
  uint64_t s = seed;
  float scale = hi - lo;
  for (int64_t i = 0; i < n; ++i) out[i] = lo + scale * sm64_unit(&s);
}

/* randn (tensor.rs:1481-1500): Box-Muller in f32, cos value first and the sin
 * value as the spare, then scaled by sigma. u1 = 1 - unit lies in (0,1]. */
void oracle_randn(float *out, int64_t n, uint64_t seed, float sigma) {
  uint64_t s = seed;
  int64_t i = 0;
  const float tau = 6.28318530717958647692f;
  while (i < n) {
    float u1 = 1.0f - sm64_unit(&s);
    float u2 = sm64_unit(&s);
    float radius = sqrtf(-2.0f * logf(u1));
    float angle = tau * u2;
    out[i++] = sigma * (radius * cosf(angle));
    if (i < n) out[i++] = sigma * (radius * sinf(angle));
  }
}

/* ----------------------------------------------------------- epilogues -- */

/* Epilogue codes, as the C ABI's MMR_EPI_*: MatMul -> optional Add(bias[N])
 * -> optional activation. */
enum {
  EPI_NONE = 0, EPI_BIAS = 1, EPI_BIAS_RELU = 2, EPI_RELU = 3,
  EPI_RELU6 = 4, EPI_BIAS_RELU6 = 5, EPI_GELU_ERF = 6, EPI_BIAS_GELU_ERF = 7,
  EPI_GELU_TANH = 8, EPI_BIAS_GELU_TANH = 9, EPI_SILU = 10, EPI_BIAS_SILU = 11
};
enum { ACT_NONE = 0, ACT_RELU = 1, ACT_RELU6 = 2, ACT_GELU_ERF = 3, ACT_GELU_TANH = 4, ACT_SILU = 5 };

static inline int epi_has_bias(int e) { return e == EPI_BIAS || e == EPI_BIAS_RELU || (e >= EPI_RELU6 && (e & 1)); }
static inline int epi_act(int e) {
  if (e == EPI_BIAS_RELU || e == EPI_RELU) return ACT_RELU;
  if (e >= EPI_RELU6 && e <= EPI_BIAS_SILU) return ACT_RELU6 + (e - EPI_RELU6) / 2;
  return ACT_NONE;
}

/* relu_f32, cpu.rs:2158-2160: NaN kept (payload too), x>0 kept, else +0. */
static inline float relu_ref(float x) {
  if (x != x) return x;
  if (x > 0.0f) return x;
  return 0.0f;
}

/* relu6_f32, cpu.rs:2161-2163. */
static inline float relu6_ref(float x) {
  if (x != x) return x;
  if (x <= 0.0f) return 0.0f;
  if (x >= 6.0f) return 6.0f;
  return x;
}

/* sigmoid_value, cpu.rs:2137-2144 (exp never overflows). Rust's f32::exp is
 * the platform libm's expf, which this calls too. */
static inline float sigmoid_ref(float x) {
  if (x >= 0.0f) return 1.0f / (1.0f + expf(-x));
  const float e = expf(x);
  return e / (1.0f + e);
}

/* silu_f32, cpu.rs:2166-2168. */
static inline float silu_ref(float x) {
  if (x == -INFINITY) return -0.0f;
  return x * sigmoid_ref(x);
}

/* gelu_tanh_approx_f32, cpu.rs:2214-2222: f32 arithmetic, libm tanhf. */
static inline float gelu_tanh_ref(float x) {
  if (x == -INFINITY) return -0.0f;
  if (x == INFINITY) return INFINITY;
  const float cubic = x * x * x;
  const float t = tanhf(0.7978846f * (x + 0.044715f * cubic));
  return 0.5f * x * (1.0f + t);
}

/* erfc of a finite nonnegative f64, cpu.rs:2031-2099: the classical rational
 * erf / erfc approximants on [0,1), [1,8), [8,27], Horner evaluation in f64
 * (horner / horner_leading_one, cpu.rs:2031-2046), exp(-x^2) from libm. */
static double horner_ref(double x, const double *c, int n) {
  double r = c[0];
  for (int i = 1; i < n; ++i) r = r * x + c[i];
  return r;
}
static double horner_one_ref(double x, const double *c, int n) {
  double r = x + c[0];
  for (int i = 1; i < n; ++i) r = r * x + c[i];
  return r;
}
static const double ERF_T[5] = {9.60497373987051638749e0, 9.00260197203842689217e1, 2.23200534594684319226e3,
                                7.00332514112805075473e3, 5.55923013010394962768e4};
static const double ERF_U[5] = {3.35617141647503099647e1, 5.21357949780152679795e2, 4.59432382970980127987e3,
                                2.26290000613890934246e4, 4.92673942608635921086e4};
static const double ERFC_P[9] = {2.46196981473530512524e-10, 5.64189564831068821977e-1, 7.46321056442269912687e0,
                                 4.86371970985681366614e1, 1.96520832956077098242e2, 5.26445194995477358631e2,
                                 9.34528527171957607540e2, 1.02755188689515710272e3, 5.57535335369399327526e2};
static const double ERFC_Q[8] = {1.32281951154744992508e1, 8.67072140885989742329e1, 3.54937778887819891062e2,
                                 9.75708501743205489753e2, 1.82390916687909736289e3, 2.24633760818710981792e3,
                                 1.65666309194161350182e3, 5.57535340817727675546e2};
static const double ERFC_R[6] = {5.64189583547755073984e-1, 1.27536670759978104416e0, 5.01905042251180477414e0,
                                 6.16021097993053585195e0, 7.40974269950448939160e0, 2.97886665372100240670e0};
static const double ERFC_S[6] = {2.26052863220117276590e0, 9.39603524938001434673e0, 1.20489539808096656605e1,
                                 1.70814450747565897222e1, 9.60896809063285878198e0, 3.36907645100081516050e0};
static double erfc_nonnegative_ref(double x) {
  if (x < 1.0) return 1.0 - x * horner_ref(x * x, ERF_T, 5) / horner_one_ref(x * x, ERF_U, 5);
  if (x > 27.0) return 0.0;
  const double fraction = x < 8.0 ? horner_ref(x, ERFC_P, 9) / horner_one_ref(x, ERFC_Q, 8)
                                  : horner_ref(x, ERFC_R, 6) / horner_one_ref(x, ERFC_S, 6);
  return exp(-x * x) * fraction;
}

/* gelu_erf_value_f32, cpu.rs:2117-2129: f64 evaluation, one rounding to f32. */
static inline float gelu_erf_ref(float x) {
  if (x != x || x == 0.0f) return x;
  if (x == -INFINITY) return -0.0f;
  if (x == INFINITY) return INFINITY;
  const double ec = erfc_nonnegative_ref(fabs((double)x) / 1.41421356237309504880);
  const double v = x < 0.0f ? 0.5 * (double)x * ec : 0.5 * (double)x * (2.0 - ec);
  return (float)v;
}

static inline float activation_ref(int act, float x) {
  switch (act) {
    case ACT_RELU: return relu_ref(x);
    case ACT_RELU6: return relu6_ref(x);
    case ACT_GELU_ERF: return gelu_erf_ref(x);
    case ACT_GELU_TANH: return gelu_tanh_ref(x);
    case ACT_SILU: return silu_ref(x);
    default: return x;
  }
}

void oracle_relu(float *x, int64_t n) {
  for (int64_t i = 0; i < n; ++i) x[i] = relu_ref(x[i]);
}

/* In-place activation of n values; act is the epilogue code's activation
 * (an MMR_EPI_* value: its bias part is ignored). Returns 1 for a bad code. */
int oracle_activation(float *x, int64_t n, int epi) {
  if (epi < EPI_NONE || epi > EPI_BIAS_SILU) return 1;
  const int act = epi_act(epi);
  for (int64_t i = 0; i < n; ++i) x[i] = activation_ref(act, x[i]);
  return 0;
}

static inline float apply_epilogue(float s, const float *bias, int64_t col, int epi) {
  if (epi_has_bias(epi)) s = s + bias[col];
  return activation_ref(epi_act(epi), s);
}

/* ------------------------------------------------------- strided GEMM -- */

typedef struct {
  int64_t batch, m, n, k;
  const float *a; int64_t a_sb, a_sm, a_sk;
  const float *b; int64_t b_sb, b_sk, b_sn;
  float *c; int64_t c_sb, c_sm, c_sn;
  const float *bias; int epi;
  const int64_t *rows; int64_t nrows; /* optional row subset; c row i <- rows[i] */
  int64_t next;                        /* work counter (row blocks) */
  pthread_mutex_t lock;
} gemm_job;

#define ORACLE_RB 4

static int64_t take_work(gemm_job *j) {
  pthread_mutex_lock(&j->lock);
  int64_t w = j->next++;
  pthread_mutex_unlock(&j->lock);
  return w;
}

/* One block of up to ORACLE_RB output rows of one batch entry. The per-element
 * arithmetic is exactly gemm_axpy_f32's: acc starts at +0 and takes
 * acc = acc + a*b for p = 0..K-1 in increasing order. */
static void gemm_row_block(gemm_job *j, int64_t bi, int64_t r0, int64_t rcount, float *acc) {
  const int64_t n = j->n, k = j->k;
  const float *a = j->a + bi * j->a_sb;
  const float *b = j->b + bi * j->b_sb;
  int64_t src_rows[ORACLE_RB];
  for (int64_t r = 0; r < rcount; ++r)
    src_rows[r] = j->rows ? j->rows[r0 + r] : r0 + r;
  memset(acc, 0, sizeof(float) * (size_t)(ORACLE_RB * n));
  for (int64_t p = 0; p < k; ++p) {
    const float *brow = b + p * j->b_sk;
    for (int64_t r = 0; r < rcount; ++r) {
      const float av = a[src_rows[r] * j->a_sm + p * j->a_sk];
      float *ar = acc + r * n;
      if (j->b_sn == 1) {
        for (int64_t col = 0; col < n; ++col) ar[col] = ar[col] + av * brow[col];
      } else {
        for (int64_t col = 0; col < n; ++col) ar[col] = ar[col] + av * brow[col * j->b_sn];
      }
    }
  }
  float *c = j->c + bi * j->c_sb;
  for (int64_t r = 0; r < rcount; ++r)
    for (int64_t col = 0; col < n; ++col)
      c[(r0 + r) * j->c_sm + col * j->c_sn] = apply_epilogue(acc[r * n + col], j->bias, col, j->epi);
}

static void *gemm_worker(void *arg) {
  gemm_job *j = (gemm_job *)arg;
  const int64_t out_rows = j->rows ? j->nrows : j->m;
  const int64_t blocks_per_batch = (out_rows + ORACLE_RB - 1) / ORACLE_RB;
  float *acc = (float *)malloc(sizeof(float) * (size_t)(ORACLE_RB * (j->n > 0 ? j->n : 1)));
  if (!acc) return (void *)1;
  for (;;) {
    int64_t w = take_work(j);
    if (w >= j->batch * blocks_per_batch) break;
    int64_t bi = w / blocks_per_batch, blk = w % blocks_per_batch;
    int64_t r0 = blk * ORACLE_RB;
    int64_t rc = out_rows - r0 < ORACLE_RB ? out_rows - r0 : ORACLE_RB;
    gemm_row_block(j, bi, r0, rc, acc);
  }
  free(acc);
  return 0;
}

static int resolve_threads(int nthreads) {
  if (nthreads > 0) return nthreads;
  long c = sysconf(_SC_NPROCESSORS_ONLN);
  return c > 0 ? (int)c : 1;
}

/* Batched strided matmul in the reference's arithmetic. Element strides are
 * given per operand for (batch, row, col); a batch stride of 0 broadcasts that
 * operand over the batch (validation.rs:2357-2388). K = 0 writes +0 (then the
 * epilogue). Rows may be subset with `rows`/`nrows` (NULL = all rows). Row
 * blocks are shared among threads; every output element is still produced by
 * one sequential K loop, so the result is independent of the thread count. */
int oracle_gemm(int64_t batch, int64_t m, int64_t n, int64_t k,
                const float *a, int64_t a_sb, int64_t a_sm, int64_t a_sk,
                const float *b, int64_t b_sb, int64_t b_sk, int64_t b_sn,
                float *c, int64_t c_sb, int64_t c_sm, int64_t c_sn,
                const float *bias, int epi, const int64_t *rows, int64_t nrows,
                int nthreads) {
  if (batch < 0 || m < 0 || n < 0 || k < 0) return 1;
  if (epi < EPI_NONE || epi > EPI_BIAS_SILU) return 3;
  if (epi_has_bias(epi) && !bias && n > 0) return 2;
  gemm_job j = {batch, m, n, k, a, a_sb, a_sm, a_sk, b, b_sb, b_sk, b_sn,
                c, c_sb, c_sm, c_sn, bias, epi, rows, nrows, 0, PTHREAD_MUTEX_INITIALIZER};
  pthread_mutex_init(&j.lock, NULL);
  int nt = resolve_threads(nthreads);
  if (nt > 256) nt = 256;
  pthread_t th[256];
  int started = 0, rc = 0;
  for (int t = 1; t < nt; ++t)
    if (pthread_create(&th[started], NULL, gemm_worker, &j) == 0) ++started;
  if (gemm_worker(&j)) rc = 3;
  for (int t = 0; t < started; ++t) {
    void *res = 0;
    pthread_join(th[t], &res);
    if (res) rc = 3;
  }
  pthread_mutex_destroy(&j.lock);
  return rc;
}

/* fp64 comparator (not the oracle): same indexing, double accumulation. Used
 * only to attribute error between the GPU result and the f32 reference. */
int oracle_gemm_f64(int64_t batch, int64_t m, int64_t n, int64_t k,
                    const float *a, int64_t a_sb, int64_t a_sm, int64_t a_sk,
                    const float *b, int64_t b_sb, int64_t b_sk, int64_t b_sn,
                    double *c, const int64_t *rows, int64_t nrows) {
  const int64_t out_rows = rows ? nrows : m;
  double *acc = (double *)malloc(sizeof(double) * (size_t)(n > 0 ? n : 1));
  if (!acc) return 3;
  for (int64_t bi = 0; bi < batch; ++bi) {
    for (int64_t i = 0; i < out_rows; ++i) {
      int64_t r = rows ? rows[i] : i;
      memset(acc, 0, sizeof(double) * (size_t)n);
      for (int64_t p = 0; p < k; ++p) {
        double av = a[bi * a_sb + r * a_sm + p * a_sk];
        const float *brow = b + bi * b_sb + p * b_sk;
        for (int64_t col = 0; col < n; ++col) acc[col] += av * (double)brow[col * b_sn];
      }
      memcpy(c + (bi * out_rows + i) * n, acc, sizeof(double) * (size_t)n);
    }
  }
  free(acc);
  return 0;
}

/* ------------------------------------------- gemm_avx2, loop structure -- */

typedef struct {
  int64_t m, n, k;
  const float *a, *b;
  float *c;
  int64_t row0, row1;
} avx2_job;

/* cpu.rs:3068-3098 restated with its loop structure: per row, per 8-column
 * block, one register accumulator over all K with _mm256_add_ps(acc,
 * _mm256_mul_ps(a, b)), one store per block, scalar tail in the same order.
 * Row-major contiguous operands only, as the reference entry requires. */
__attribute__((target("avx2"))) static void gemm_avx2_rows(const avx2_job *j) {
  const int64_t n = j->n, k = j->k;
  for (int64_t row = j->row0; row < j->row1; ++row) {
    int64_t col = 0;
    while (n - col >= 8) {
      __m256 acc = _mm256_setzero_ps();
      for (int64_t p = 0; p < k; ++p) {
        __m256 av = _mm256_set1_ps(j->a[row * k + p]);
        __m256 bv = _mm256_loadu_ps(j->b + p * n + col);
        acc = _mm256_add_ps(acc, _mm256_mul_ps(av, bv));
      }
      _mm256_storeu_ps(j->c + row * n + col, acc);
      col += 8;
    }
    while (col < n) {
      float acc = 0.0f;
      for (int64_t p = 0; p < k; ++p) acc += j->a[row * k + p] * j->b[p * n + col];
      j->c[row * n + col] = acc;
      col += 1;
    }
  }
}

static void *avx2_worker(void *arg) {
  gemm_avx2_rows((const avx2_job *)arg);
  return 0;
}

/* Row-sharded over `nthreads` host threads (0 = all online cores). Each output
 * element is independent, so this is bitwise identical to one thread. Rows
 * [row0, row1) of C are computed; A, B, C are the full row-major matrices. */
int oracle_gemm_avx2_restated(int64_t m, int64_t n, int64_t k, const float *a,
                              const float *b, float *c, int64_t row0, int64_t row1,
                              int nthreads) {
  if (row0 < 0 || row1 > m || row0 > row1) return 1;
  int nt = resolve_threads(nthreads);
  if (nt > 256) nt = 256;
  int64_t rows = row1 - row0;
  if (nt > rows && rows > 0) nt = (int)rows;
  if (nt < 1) nt = 1;
  avx2_job jobs[256];
  pthread_t th[256];
  int64_t per = (rows + nt - 1) / nt;
  int started = 0;
  for (int t = 0; t < nt; ++t) {
    avx2_job jb = {m, n, k, a, b, c, row0 + t * per, row0 + (t + 1) * per};
    if (jb.row1 > row1) jb.row1 = row1;
    if (jb.row0 > jb.row1) jb.row0 = jb.row1;
    jobs[t] = jb;
  }
  int spawned[256] = {0};
  for (int t = 1; t < nt; ++t) {
    if (pthread_create(&th[t], NULL, avx2_worker, &jobs[t]) == 0) { spawned[t] = 1; ++started; }
    else gemm_avx2_rows(&jobs[t]);
  }
  gemm_avx2_rows(&jobs[0]);
  for (int t = 1; t < nt; ++t)
    if (spawned[t]) pthread_join(th[t], NULL);
  return 0;
}

/* ---------------------------------------------------- known answers -- */

/* cpu.rs:827-846: A=[[1,2,3],[4,5,6]], B=[[7,8],[9,10],[11,12]] ->
 * [58,64,139,154] exactly. Returns 0 on success. */
int oracle_selfcheck_kat(void) {
  const float a[6] = {1, 2, 3, 4, 5, 6};
  const float b[6] = {7, 8, 9, 10, 11, 12};
  const float want[4] = {58, 64, 139, 154};
  float out[4];
  for (int i = 0; i < 4; ++i) out[i] = NAN;
  if (oracle_gemm(1, 2, 2, 3, a, 0, 3, 1, b, 0, 2, 1, out, 0, 2, 1, 0, EPI_NONE, 0, 0, 1)) return 1;
  if (memcmp(out, want, sizeof out)) return 2;
  for (int i = 0; i < 4; ++i) out[i] = NAN;
  if (oracle_gemm_avx2_restated(2, 2, 3, a, b, out, 0, 2, 1)) return 3;
  if (memcmp(out, want, sizeof out)) return 4;
  return 0;
}
